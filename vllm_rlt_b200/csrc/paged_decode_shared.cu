// Paged decode attention that reads pages shared by several rows once.
//
// With prefix caching (vllm_rlt/core/kv_cache_manager.py:211-251: complete
// prompt pages are published by content hash and handed to later requests
// by reference, `_refs[b] += 1`), many rows of a decode batch point their
// tables at the same physical pages for a common prompt prefix. The plain
// decode kernel reads those pages once per row. Here a host-built plan cuts
// the work into chunks: a chunk is a token range of one table row together
// with the rows (members) that share it. One CTA reads each 32-token sub-tile
// of its chunk once and runs the online softmax of every (member row, query
// head) pair of its KV head on it, writing an fp32 partial (o, max, sum) per
// pair. Each row's own tokens after the shared prefix go through the plain
// decode kernel first (rlt_paged_decode_lse on per-row suffix tables), which
// leaves the suffix result in `out` and its log-sum-exp in `suffix_lse`; a
// merge kernel then folds the prefix partials into `out`. Result = softmax(q K^T * scale) V over
// the row's context, the semantics of torch_paged_attention
// (vllm_rlt/kernels/paged_attention.py:12-36).
//
// Plan arrays (device int32): chunks[c] = {table_row, token_begin, token_end,
// member_begin, member_count}; members[member_begin + i] = row id;
// member_slots[...] = the partial slot of that (row, chunk); row_slots[r] ..
// row_slots[r+1] = the slots of row r. member_count * (Hq / Hkv) <= 32.
#include <type_traits>

#include "common.cuh"

namespace rlt {
namespace {

constexpr int kSubTile = 32;   // tokens per shared-memory sub-tile (one per lane)
constexpr int kMaxPairs = 32;  // (member, query head) pairs per CTA
constexpr int kWarps = 4;
constexpr int kPairsPerWarp = kMaxPairs / kWarps;
constexpr int kPhaseChunks = 1;  // the prefix-chunk partials
constexpr int kPhaseMerge = 2;   // their merge into the suffix result

struct SharedParams {
  const void* q;
  const void* k;
  const void* v;
  const int32_t* tables;
  const int32_t* chunks;
  const int32_t* members;
  const int32_t* member_slots;
  float* ws_o;   // [slots, Hq, D]
  float* ws_ml;  // [slots, Hq, 2]
  int32_t* status;
  int hq, hkv, group, page, width, num_rows, num_slots, num_members;
  int64_t num_blocks;
  int64_t q_rs, q_hs, k_bs, k_ts, k_hs, v_bs, v_ts, v_hs, t_rs;
  float scale_log2;
};

template <int D>
struct SharedLayout {
  static constexpr int kRowFloats = D + 4;  // fp32 row + 16 B pad: conflict-free per-token reads
  static constexpr int kBytes = (kMaxPairs * D + 2 * kSubTile * kRowFloats) * 4;
};

template <typename T, int D>
__global__ void __launch_bounds__(kWarps * 32, 4) shared_range_kernel(const SharedParams p) {
  constexpr int kRow = SharedLayout<D>::kRowFloats;
  constexpr int kE = D / 32;                      // output dims per lane
  constexpr int kVec = 16 / sizeof(T);            // elements per 16-byte vector
  constexpr int kVecPerRow = D / kVec;
  extern __shared__ float4 smem4[];
  float* sq = reinterpret_cast<float*>(smem4);    // [kMaxPairs][D], pre-scaled q
  float* sk = sq + kMaxPairs * D;                 // [kSubTile][kRow]
  float* sv = sk + kSubTile * kRow;

  const int* c = p.chunks + blockIdx.x * 5;
  const int table_row = c[0], tok_begin = c[1], tok_end = c[2];
  const int member_begin = c[3], member_count = c[4];
  const int kvh = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pairs = member_count * p.group;
  if (pairs <= 0 || pairs > kMaxPairs || tok_begin >= tok_end || table_row < 0 ||
      table_row >= p.num_rows || member_begin < 0 || member_begin + member_count > p.num_members) {
    if (tid == 0 && pairs != 0) raise_status(p.status, kStatusBadSequence);
    return;
  }

  // q of every pair (member i, head j of this KV head), scaled to base 2
  for (int e = tid; e < pairs * D; e += kWarps * 32) {
    const int pair = e / D, d = e % D;
    const int row = p.members[member_begin + pair / p.group];
    const int qh = kvh * p.group + pair % p.group;
    float x = 0.f;
    if (row >= 0 && row < p.num_rows)
      x = to_f32<T>(static_cast<const T*>(p.q)[row * p.q_rs + qh * p.q_hs + d]);
    sq[e] = x * p.scale_log2;
  }

  float m[kPairsPerWarp], l[kPairsPerWarp], o[kPairsPerWarp][kE];
#pragma unroll
  for (int i = 0; i < kPairsPerWarp; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int e = 0; e < kE; ++e) o[i][e] = 0.f;
  }

  const T* kbase = static_cast<const T*>(p.k) + kvh * p.k_hs;
  const T* vbase = static_cast<const T*>(p.v) + kvh * p.v_hs;
  for (int t0 = tok_begin; t0 < tok_end; t0 += kSubTile) {
    __syncthreads();  // q staged / previous sub-tile consumed
    for (int e = tid; e < 2 * kSubTile * kVecPerRow; e += kWarps * 32) {
      const bool is_v = e >= kSubTile * kVecPerRow;
      const int idx = is_v ? e - kSubTile * kVecPerRow : e;
      const int tok = idx / kVecPerRow, vec = idx % kVecPerRow;
      const int pos = t0 + tok;
      float f[kVec];
#pragma unroll
      for (int i = 0; i < kVec; ++i) f[i] = 0.f;
      const int pg = pos / p.page;
      if (pos < tok_end && pg >= p.width) {
        if (vec == 0) raise_status(p.status, kStatusBadLength);
      } else if (pos < tok_end) {
        const int b = p.tables[table_row * p.t_rs + pg];
        if (b >= 0 && b < p.num_blocks) {
          const T* src = (is_v ? vbase + b * p.v_bs + (pos % p.page) * p.v_ts
                               : kbase + b * p.k_bs + (pos % p.page) * p.k_ts) +
                         vec * kVec;
          unpack16<T>(ld_stream(src), f);
        } else if (vec == 0) {
          raise_status(p.status, kStatusBadBlock);
        }
      }
      float* dst = (is_v ? sv : sk) + tok * kRow + vec * kVec;
#pragma unroll
      for (int i = 0; i < kVec; i += 4)
        *reinterpret_cast<float4*>(dst + i) = make_float4(f[i], f[i + 1], f[i + 2], f[i + 3]);
    }
    __syncthreads();
    const int valid = min(kSubTile, tok_end - t0);

#pragma unroll
    for (int i = 0; i < kPairsPerWarp; ++i) {
      const int pair = warp + kWarps * i;
      if (pair >= pairs) break;  // warp-uniform
      // score of token `lane`
      const float* qv = sq + pair * D;
      const float* kr = sk + lane * kRow;
      float s = 0.f;
#pragma unroll 8
      for (int d = 0; d < D; d += 4) {
        const float4 a = *reinterpret_cast<const float4*>(qv + d);
        const float4 b = *reinterpret_cast<const float4*>(kr + d);
        s = fmaf(a.x, b.x, s);
        s = fmaf(a.y, b.y, s);
        s = fmaf(a.z, b.z, s);
        s = fmaf(a.w, b.w, s);
      }
      s = lane < valid ? s : -INFINITY;
      float mt = s;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(kFullMask, mt, off));
      const float m_new = fmaxf(m[i], mt);
      const float corr = ex2(m[i] - m_new);
      const float pr = lane < valid ? ex2(s - m_new) : 0.f;
      float ps = pr;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(kFullMask, ps, off);
      l[i] = l[i] * corr + ps;
      m[i] = m_new;
#pragma unroll
      for (int e = 0; e < kE; ++e) o[i][e] *= corr;
      for (int t = 0; t < valid; ++t) {
        const float pt = __shfl_sync(kFullMask, pr, t);
        const float* vr = sv + t * kRow + lane * kE;
        if constexpr (kE == 4) {
          const float4 vv = *reinterpret_cast<const float4*>(vr);
          o[i][0] = fmaf(pt, vv.x, o[i][0]);
          o[i][1] = fmaf(pt, vv.y, o[i][1]);
          o[i][2] = fmaf(pt, vv.z, o[i][2]);
          o[i][3] = fmaf(pt, vv.w, o[i][3]);
        } else {
#pragma unroll
          for (int e = 0; e < kE; ++e) o[i][e] = fmaf(pt, vr[e], o[i][e]);
        }
      }
    }
  }

#pragma unroll
  for (int i = 0; i < kPairsPerWarp; ++i) {
    const int pair = warp + kWarps * i;
    if (pair >= pairs) break;
    const int slot = p.member_slots[member_begin + pair / p.group];
    if (slot < 0 || slot >= p.num_slots) {
      if (lane == 0) raise_status(p.status, kStatusBadSequence);
      continue;
    }
    const int qh = kvh * p.group + pair % p.group;
    float* dst = p.ws_o + (static_cast<int64_t>(slot) * p.hq + qh) * D + lane * kE;
#pragma unroll
    for (int e = 0; e < kE; ++e) dst[e] = o[i][e];
    if (lane == 0) {
      float* ml = p.ws_ml + (static_cast<int64_t>(slot) * p.hq + qh) * 2;
      ml[0] = m[i];
      ml[1] = l[i];
    }
  }
}

// 16-bit K/V on the tensor cores (mma.sync m16n8k16, fp32 accumulate): a
// chunk has at most 32 (member, query head) pairs, one or two 16-row M tiles,
// far below the 64/128 rows of a tcgen05 tile. The CTA stages 64-token K/V
// sub-tiles in shared memory (cp.async, double buffered: the next sub-tile is
// in flight while one is consumed -- a third buffer measured no faster alone
// and slowed the suffix decode that runs beside this kernel; rows padded to an
// odd number of 16-byte units so ldmatrix reads are conflict-free). Warp w takes M
// tile w % tiles and a slice of every sub-tile's tokens: S = Q K^T (Q
// fragments stay in registers for the whole chunk, K fragments by ldmatrix),
// base-2 online softmax on the S fragments (a row's values sit in the 4 lanes
// of a quad), P rounded to the input type and reused in registers as the A
// operand of O += P V (V fragments by ldmatrix.trans). The warps of one M tile
// merge their token slices through shared memory at the end.
template <int D>
struct LayoutMma {
  static constexpr int kTokens = 64;                      // tokens per staged sub-tile
  static constexpr int kRowBytes = D * 2 + 16;            // padded 16-bit row
  static constexpr int kTileBytes = kTokens * kRowBytes;  // one K or V sub-tile
  static constexpr int kQBytes = kMaxPairs * kRowBytes;
  static constexpr int kBytes = kQBytes + 2 * 2 * kTileBytes;  // Q + 2 buffers x (K, V)
  // token-slice merge, reusing the K/V staging: [warp][16 rows][D + 2] floats
  static constexpr int kCombineBytes = kWarps * 16 * (D + 2) * 4;
  static_assert(kCombineBytes <= 2 * 2 * kTileBytes, "merge buffer exceeds the K/V staging");
  static_assert(2 * (kBytes + 1024) <= 228 * 1024, "two CTAs per SM");
  static_assert((kRowBytes / 16) % 2 == 1, "ldmatrix rows must be an odd number of 16-byte units");
};

__device__ __forceinline__ uint32_t smem_addr(const void* ptr) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(ptr));
}

// 16-byte global -> shared copy; src_bytes 0 writes zeros (nothing is read)
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack_pair<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack_pair<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <typename T, int D>
__global__ void __launch_bounds__(kWarps * 32, 2) shared_range_mma_kernel(const SharedParams p) {
  using L = LayoutMma<D>;
  constexpr int kKSteps = D / 16;  // k16 steps over the head dim (S = Q K^T)
  constexpr int kDTiles = D / 8;   // n8 tiles over the head dim (O)
  constexpr int kRowVecs = D / 8;  // 16-byte vectors per row
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* sq = smem;
  uint8_t* skv = smem + L::kQBytes;  // [buffer][K, V][token][padded row]

  const int* c = p.chunks + blockIdx.x * 5;
  const int table_row = c[0], tok_begin = c[1], tok_end = c[2];
  const int member_begin = c[3], member_count = c[4];
  const int kvh = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pairs = member_count * p.group;
  if (pairs <= 0 || pairs > kMaxPairs || tok_begin >= tok_end || table_row < 0 ||
      table_row >= p.num_rows || member_begin < 0 || member_begin + member_count > p.num_members) {
    if (tid == 0 && pairs != 0) raise_status(p.status, kStatusBadSequence);
    return;
  }
  const int tiles = pairs <= 16 ? 1 : 2;
  const int slices = kWarps / tiles;  // 4 or 2 token slices per sub-tile
  const int mt = warp % tiles, sl = warp / tiles;
  const int slice_tokens = L::kTokens / slices;  // 16 or 32
  const int g = lane >> 2, tig = lane & 3;

  // Q of every pair, in the input type (rows >= pairs stay zero)
  for (int e = tid; e < kMaxPairs * kRowVecs; e += kWarps * 32) {
    const int row = e / kRowVecs, v = e % kRowVecs;
    uint32_t w[4] = {0, 0, 0, 0};
    if (row < pairs) {
      const int r = p.members[member_begin + row / p.group];
      const int qh = kvh * p.group + row % p.group;
      if (r >= 0 && r < p.num_rows) {
        const T* src = static_cast<const T*>(p.q) + r * p.q_rs + qh * p.q_hs + v * 8;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          T two[2] = {src[2 * i], src[2 * i + 1]};
          w[i] = *reinterpret_cast<uint32_t*>(two);
        }
      }
    }
    *reinterpret_cast<uint4*>(sq + row * L::kRowBytes + v * 16) = make_uint4(w[0], w[1], w[2], w[3]);
  }

  const T* kbase = static_cast<const T*>(p.k) + kvh * p.k_hs;
  const T* vbase = static_cast<const T*>(p.v) + kvh * p.v_hs;
  auto tile_ptr = [&](int buf, int which) { return skv + (buf * 2 + which) * L::kTileBytes; };
  // Loader: 4 threads per token copy its K row and its V row, each thread a
  // quarter of both (vector j * 4 + quarter, so the 4 threads of a token read
  // 64 contiguous bytes per copy); a pass of the CTA covers kPassTokens
  // tokens. A thread keeps the page index and in-page offset of each of its
  // tokens and steps them by one sub-tile per call, so a copy costs no
  // division: per token one address, then 2 x kVecs copies. The page ids a
  // sub-tile's copies need are read when the previous sub-tile's copies are
  // issued, so the table's round trip never sits between a warp and its math.
  constexpr int kThreads = kWarps * 32;
  constexpr int kQuarter = 4;
  constexpr int kVecs = kRowVecs / kQuarter;  // 16-byte vectors per thread per row
  constexpr int kPassTokens = kThreads / kQuarter;
  constexpr int kPasses = L::kTokens / kPassTokens;
  static_assert(kRowVecs % kQuarter == 0 && L::kTokens % kPassTokens == 0, "loader mapping");
  const int quarter = tid % kQuarter, ltok = tid / kQuarter;
  const int64_t trow = static_cast<int64_t>(table_row) * p.t_rs;
  const int step_pages = L::kTokens / p.page, step_off = L::kTokens % p.page;
  int pg[kPasses], off[kPasses];  // position of token ltok + i * kPassTokens of the next sub-tile
  int blk[kPasses];               // its page id; INT32_MIN: nothing to read
#pragma unroll
  for (int i = 0; i < kPasses; ++i) {
    const int pos = tok_begin + ltok + i * kPassTokens;
    pg[i] = pos / p.page;
    off[i] = pos % p.page;
  }
  auto read_ids = [&](int t0) {
#pragma unroll
    for (int i = 0; i < kPasses; ++i) {
      blk[i] = INT32_MIN;  // past the chunk or past the table
      if (t0 + ltok + i * kPassTokens < tok_end) {
        if (pg[i] < p.width) {
          blk[i] = p.tables[trow + pg[i]];
        } else if (quarter == 0) {
          raise_status(p.status, kStatusBadLength);
        }
      }
    }
  };
  auto load_tile = [&](int buf, int t0) {  // t0: tok_begin, then one sub-tile further per call
#pragma unroll
    for (int i = 0; i < kPasses; ++i) {
      const int tok = ltok + i * kPassTokens;
      const int b = blk[i];
      const T* ks = kbase;  // any valid address when nothing is read
      const T* vs = vbase;
      uint32_t bytes = 0;
      if (b >= 0 && b < p.num_blocks) {
        ks = kbase + b * p.k_bs + off[i] * p.k_ts + quarter * 8;
        vs = vbase + b * p.v_bs + off[i] * p.v_ts + quarter * 8;
        bytes = 16;
      } else if (b != INT32_MIN && quarter == 0) {
        raise_status(p.status, kStatusBadBlock);
      }
      const uint32_t kd = smem_addr(tile_ptr(buf, 0) + tok * L::kRowBytes + quarter * 16);
      const uint32_t vd = smem_addr(tile_ptr(buf, 1) + tok * L::kRowBytes + quarter * 16);
#pragma unroll
      for (int j = 0; j < kVecs; ++j) {
        cp_async16(kd + j * kQuarter * 16, ks + (bytes ? j * kQuarter * 8 : 0), bytes);
        cp_async16(vd + j * kQuarter * 16, vs + (bytes ? j * kQuarter * 8 : 0), bytes);
      }
      pg[i] += step_pages;
      off[i] += step_off;
      if (off[i] >= p.page) {
        off[i] -= p.page;
        ++pg[i];
      }
    }
    cp_async_commit();
    read_ids(t0 + L::kTokens);
  };
  read_ids(tok_begin);
  load_tile(0, tok_begin);
  __syncthreads();  // Q staged

  // Q fragments of this warp's M tile (matrix j = lane / 8: rows +8 for odd j,
  // columns +8 for j >= 2)
  uint32_t qa[kKSteps][4];
  {
    const int j = lane >> 3, r = lane & 7;
    const uint8_t* base = sq + (mt * 16 + r + 8 * (j & 1)) * L::kRowBytes + 16 * (j >> 1);
#pragma unroll
    for (int ks = 0; ks < kKSteps; ++ks)
      ldsm_x4(smem_addr(base + ks * 32), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
  }

  float o[kDTiles][4];
#pragma unroll
  for (int n = 0; n < kDTiles; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};

  int buf = 0;
  for (int t0 = tok_begin; t0 < tok_end; t0 += L::kTokens, buf ^= 1) {
    if (t0 + L::kTokens < tok_end) {
      load_tile(buf ^ 1, t0 + L::kTokens);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // this sub-tile's K and V are in shared memory

    const uint8_t* ktile = tile_ptr(buf, 0);
    const uint8_t* vtile = tile_ptr(buf, 1);
    const int tok0 = sl * slice_tokens;
    float s[4][4];  // up to 4 n8 token tiles
#pragma unroll
    for (int j = 0; j < 4; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
    {
      // B fragments of K: matrix jj = lane / 8 -> token tile +(jj >> 1), dims +8 (jj & 1)
      const int jj = lane >> 3, r = lane & 7;
#pragma unroll
      for (int ks = 0; ks < kKSteps; ++ks) {
#pragma unroll
        for (int j = 0; j < 4; j += 2) {
          if (j * 8 >= slice_tokens) break;
          const uint8_t* a = ktile + (tok0 + (j + (jj >> 1)) * 8 + r) * L::kRowBytes + ks * 32 +
                             16 * (jj & 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(smem_addr(a), b0, b1, b2, b3);
          mma16816<T>(s[j], qa[ks], b0, b1);
          mma16816<T>(s[j + 1], qa[ks], b2, b3);
        }
      }
    }
    // scale, mask the tokens past the chunk, online softmax of rows g and g + 8
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (j * 8 >= slice_tokens) break;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tk = t0 + tok0 + j * 8 + 2 * tig + (e & 1);
        s[j][e] = tk < tok_end ? s[j][e] * p.scale_log2 : -INFINITY;
        mx[e >> 1] = fmaxf(mx[e >> 1], s[j][e]);
      }
    }
    float corr[2], mref[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(kFullMask, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(kFullMask, mx[h], 2));
      const float m_new = fmaxf(mrow[h], mx[h]);
      mref[h] = m_new == -INFINITY ? 0.f : m_new;
      corr[h] = ex2(mrow[h] - mref[h]);
      mrow[h] = m_new;
      lrow[h] *= corr[h];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (j * 8 >= slice_tokens) break;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        s[j][e] = ex2(s[j][e] - mref[e >> 1]);
        lrow[e >> 1] += s[j][e];
      }
    }
    // once the row maxima settle every factor is exactly 1: skip the rescale
    if (__any_sync(kFullMask, corr[0] != 1.f || corr[1] != 1.f)) {
#pragma unroll
      for (int n = 0; n < kDTiles; ++n) {
        o[n][0] *= corr[0];
        o[n][1] *= corr[0];
        o[n][2] *= corr[1];
        o[n][3] *= corr[1];
      }
    }
    // O += P V over the slice's tokens, 16 at a time
    {
      const int jj = lane >> 3, r = lane & 7;
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        if (kk * 16 >= slice_tokens) break;
        uint32_t a[4];
        a[0] = pack_pair<T>(s[2 * kk][0], s[2 * kk][1]);
        a[1] = pack_pair<T>(s[2 * kk][2], s[2 * kk][3]);
        a[2] = pack_pair<T>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
        a[3] = pack_pair<T>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
        // matrix jj: tokens +8 (jj & 1), dim tile +(jj >> 1)
        const uint8_t* vrow = vtile + (tok0 + kk * 16 + 8 * (jj & 1) + r) * L::kRowBytes;
#pragma unroll
        for (int n = 0; n < kDTiles; n += 2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(smem_addr(vrow + (n + (jj >> 1)) * 16), b0, b1, b2, b3);
          mma16816<T>(o[n], a, b0, b1);
          mma16816<T>(o[n + 1], a, b2, b3);
        }
      }
    }
    __syncthreads();  // every warp is done with this buffer before it is refilled
  }

#pragma unroll
  for (int h = 0; h < 2; ++h) {
    lrow[h] += __shfl_xor_sync(kFullMask, lrow[h], 1);
    lrow[h] += __shfl_xor_sync(kFullMask, lrow[h], 2);
  }
  // merge the token slices of each M tile (the K/V staging is free now)
  float* cb = reinterpret_cast<float*>(skv);
  {
    float* mine = cb + warp * 16 * (D + 2);
#pragma unroll
    for (int n = 0; n < kDTiles; ++n) {
      const int col = n * 8 + 2 * tig;
      mine[g * (D + 2) + col] = o[n][0];
      mine[g * (D + 2) + col + 1] = o[n][1];
      mine[(g + 8) * (D + 2) + col] = o[n][2];
      mine[(g + 8) * (D + 2) + col + 1] = o[n][3];
    }
    if (tig == 0) {
      mine[g * (D + 2) + D] = mrow[0];
      mine[g * (D + 2) + D + 1] = lrow[0];
      mine[(g + 8) * (D + 2) + D] = mrow[1];
      mine[(g + 8) * (D + 2) + D + 1] = lrow[1];
    }
  }
  __syncthreads();
  if (sl != 0) return;
  // warp (slice 0, tile mt): lane covers rows g, g + 8 and its columns
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = g + 8 * h;
    const int pair = mt * 16 + row;
    float mxs = -INFINITY;
    for (int k = 0; k < slices; ++k)
      mxs = fmaxf(mxs, cb[((k * tiles + mt) * 16 + row) * (D + 2) + D]);
    const float mref = mxs == -INFINITY ? 0.f : mxs;
    float wk[kWarps];
    float lsum = 0.f;
    for (int k = 0; k < slices; ++k) {
      const float* st = cb + ((k * tiles + mt) * 16 + row) * (D + 2);
      wk[k] = ex2(st[D] - mref);
      lsum += st[D + 1] * wk[k];
    }
    if (pair >= pairs) continue;
    const int slot = p.member_slots[member_begin + pair / p.group];
    if (slot < 0 || slot >= p.num_slots) {
      if (tig == 0) raise_status(p.status, kStatusBadSequence);
      continue;
    }
    const int qh = kvh * p.group + pair % p.group;
    float* dst = p.ws_o + (static_cast<int64_t>(slot) * p.hq + qh) * D;
#pragma unroll
    for (int n = 0; n < kDTiles; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int col = n * 8 + 2 * tig + e;
        float acc = 0.f;
        for (int k = 0; k < slices; ++k)
          acc = fmaf(cb[((k * tiles + mt) * 16 + row) * (D + 2) + col], wk[k], acc);
        dst[col] = acc;
      }
    }
    if (tig == 0) {
      float* ml = p.ws_ml + (static_cast<int64_t>(slot) * p.hq + qh) * 2;
      ml[0] = mxs;
      ml[1] = lsum;
    }
  }
}

// On entry out[row, qh] holds the row's suffix attention O_x (normalised, the
// decode kernel's result over the tokens after the shared prefix) and
// suffix_lse its base-2 log-sum-exp x; the prefix partials (o_s, m_s, l_s)
// are merged in: out = (sum_s o_s 2^(m_s - M) + O_x 2^(x - M)) /
// (sum_s l_s 2^(m_s - M) + 2^(x - M)), M the largest exponent. Each lane reads
// and rewrites only its own dims.
template <typename T, int D>
__global__ void __launch_bounds__(kWarps * 32) shared_merge_kernel(
    const float* ws_o, const float* ws_ml, const int32_t* row_slots, const float* suffix_lse,
    void* out, int hq, int num_slots, int64_t o_rs, int64_t o_hs) {
  constexpr int kE = D / 32;
  const int row = blockIdx.x;
  const int qh = blockIdx.y * kWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (qh >= hq) return;
  const int s0 = max(0, row_slots[row]), s1 = min(num_slots, row_slots[row + 1]);
  if (s1 <= s0) return;  // no shared prefix: out already holds the result
  const float x = suffix_lse[static_cast<int64_t>(row) * hq + qh];
  float mx = x;
  for (int s = s0; s < s1; ++s) mx = fmaxf(mx, ws_ml[(static_cast<int64_t>(s) * hq + qh) * 2]);
  T* dst = static_cast<T*>(out) + row * o_rs + qh * o_hs + lane * kE;
  float acc[kE];
  float den = 0.f;
  const float wx = x == -INFINITY ? 0.f : ex2(x - mx);
#pragma unroll
  for (int e = 0; e < kE; ++e) acc[e] = wx * to_f32<T>(dst[e]);
  den += wx;
  for (int s = s0; s < s1; ++s) {
    const float* ml = ws_ml + (static_cast<int64_t>(s) * hq + qh) * 2;
    if (ml[1] <= 0.f) continue;
    const float w = ex2(ml[0] - mx);
    den += ml[1] * w;
    const float* src = ws_o + (static_cast<int64_t>(s) * hq + qh) * D + lane * kE;
#pragma unroll
    for (int e = 0; e < kE; ++e) acc[e] = fmaf(src[e], w, acc[e]);
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
#pragma unroll
  for (int e = 0; e < kE; ++e) dst[e] = from_f32<T>(acc[e] * inv);
}

// Per call, from the call's own tables and lengths: row r's suffix table is
// its table shifted past its prefix_pages[r] shared pages (padded with -1)
// and its suffix length what its context holds beyond them. A row whose
// context no longer covers its shared pages is outside the plan: it is
// flagged and gets an empty suffix.
__global__ void __launch_bounds__(256) shared_suffix_kernel(
    const int32_t* __restrict__ tables, const int32_t* __restrict__ lengths,
    const int32_t* __restrict__ prefix_pages, int32_t* __restrict__ suffix_tables,
    int32_t* __restrict__ suffix_lengths, int32_t* status, int width, int page, int64_t t_rs) {
  const int r = blockIdx.x;
  int skip = prefix_pages[r];
  const int len = lengths[r];
  const bool ok = skip >= 0 && skip <= width && len >= 0 &&
                  static_cast<int64_t>(len) >= static_cast<int64_t>(skip) * page;
  if (!ok) skip = width;
  for (int j = threadIdx.x; j < width; j += blockDim.x)
    suffix_tables[static_cast<int64_t>(r) * width + j] =
        j + skip < width ? tables[r * t_rs + j + skip] : -1;
  if (threadIdx.x == 0) {
    suffix_lengths[r] = ok ? len - skip * page : 0;
    if (!ok) raise_status(status, kStatusBadLength);
  }
}

size_t workspace_bytes(int64_t slots, int hq, int d) {
  return static_cast<size_t>(slots) * hq * (d + 2) * sizeof(float);
}

template <typename T, int D>
int launch(const SharedParams& p, int num_chunks, const int32_t* row_slots,
           const float* suffix_lse, void* out, int64_t o_rs, int64_t o_hs, int phases,
           cudaStream_t stream) {
  if (!(phases & kPhaseChunks)) {
    // merge only
  } else if constexpr (std::is_same<T, float>::value) {
    constexpr int bytes = SharedLayout<D>::kBytes;
    static cudaError_t attr = cudaFuncSetAttribute(
        shared_range_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (attr != cudaSuccess) return static_cast<int>(attr);
    if (num_chunks > 0)
      shared_range_kernel<T, D><<<dim3(num_chunks, p.hkv), kWarps * 32, bytes, stream>>>(p);
  } else {
    constexpr int bytes = LayoutMma<D>::kBytes;
    static cudaError_t attr = cudaFuncSetAttribute(
        shared_range_mma_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (attr != cudaSuccess) return static_cast<int>(attr);
    if (num_chunks > 0)
      shared_range_mma_kernel<T, D><<<dim3(num_chunks, p.hkv), kWarps * 32, bytes, stream>>>(p);
  }
  if ((phases & kPhaseMerge) && p.num_rows > 0)
    shared_merge_kernel<T, D><<<dim3(p.num_rows, ceil_div(p.hq, kWarps)), kWarps * 32, 0, stream>>>(
        p.ws_o, p.ws_ml, row_slots, suffix_lse, out, p.hq, p.num_slots, o_rs, o_hs);
  return launch_status(cudaGetLastError());
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace
}  // namespace rlt

using namespace rlt;

extern "C" size_t rlt_paged_decode_shared_workspace_bytes(int32_t num_slots, int32_t num_q_heads,
                                                          int32_t head_dim) {
  if (num_slots < 0 || num_q_heads <= 0 || head_dim <= 0) return 0;
  return workspace_bytes(num_slots, num_q_heads, head_dim);
}

extern "C" int rlt_shared_prefix_suffix(const int32_t* block_tables, const int32_t* context_lengths,
                                        const int32_t* prefix_pages, int32_t* suffix_tables,
                                        int32_t* suffix_lengths, int32_t* status,
                                        int32_t num_rows, int32_t table_width, int32_t page_size,
                                        int64_t table_row_stride, void* stream) {
  if (num_rows < 0 || table_width < 0 || page_size <= 0 || table_row_stride < table_width)
    return RLT_E_SHAPE;
  if (num_rows == 0) return RLT_OK;
  shared_suffix_kernel<<<num_rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      block_tables, context_lengths, prefix_pages, suffix_tables, suffix_lengths, status,
      table_width, page_size, table_row_stride);
  return launch_status(cudaGetLastError());
}

namespace {
int shared_entry(
    const void* q, const void* key_cache, const void* value_cache, const int32_t* block_tables,
    const int32_t* chunks, const int32_t* members, const int32_t* member_slots,
    const int32_t* row_slots, const float* suffix_lse, void* out, void* workspace,
    size_t workspace_size, int32_t* status,
    int32_t dtype, int32_t num_rows, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
    int32_t page_size, int32_t table_width, int64_t num_blocks, int32_t num_chunks,
    int32_t num_slots, int32_t num_members, int64_t q_row_stride, int64_t q_head_stride, int64_t k_block_stride,
    int64_t k_token_stride, int64_t k_head_stride, int64_t v_block_stride, int64_t v_token_stride,
    int64_t v_head_stride, int64_t table_row_stride, int64_t out_row_stride,
    int64_t out_head_stride, float scale, int32_t phases, void* stream) {
  if (phases < 1 || phases > 3) return RLT_E_SHAPE;
  if (dtype != RLT_F32 && dtype != RLT_F16 && dtype != RLT_BF16) return RLT_E_DTYPE;
  if (head_dim != 64 && head_dim != 128) return RLT_E_HEAD_DIM;
  if (num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0 ||
      num_q_heads / num_kv_heads > kMaxPairs)
    return RLT_E_HEADS;
  if (num_rows < 0 || page_size <= 0 || table_width < 0 || num_blocks < 0 || num_chunks < 0 ||
      num_slots < 0 || num_members < 0)
    return RLT_E_SHAPE;
  if (workspace_size < workspace_bytes(num_slots, num_q_heads, head_dim) ||
      (num_slots > 0 && workspace == nullptr))
    return RLT_E_WORKSPACE;
  if (suffix_lse == nullptr && num_rows > 0 && (phases & kPhaseMerge)) return RLT_E_SHAPE;
  const int elt = dtype == RLT_F32 ? 4 : 2;
  if (!aligned16(key_cache) || !aligned16(value_cache) || !aligned16(workspace) ||
      (k_block_stride * elt) % 16 || (k_token_stride * elt) % 16 || (k_head_stride * elt) % 16 ||
      (v_block_stride * elt) % 16 || (v_token_stride * elt) % 16 || (v_head_stride * elt) % 16)
    return RLT_E_ALIGN;

  SharedParams p{};
  p.q = q;
  p.k = key_cache;
  p.v = value_cache;
  p.tables = block_tables;
  p.chunks = chunks;
  p.members = members;
  p.member_slots = member_slots;
  p.ws_o = static_cast<float*>(workspace);
  p.ws_ml = p.ws_o + static_cast<int64_t>(num_slots) * num_q_heads * head_dim;
  p.status = status;
  p.hq = num_q_heads;
  p.hkv = num_kv_heads;
  p.group = num_q_heads / num_kv_heads;
  p.page = page_size;
  p.width = table_width;
  p.num_rows = num_rows;
  p.num_slots = num_slots;
  p.num_members = num_members;
  p.num_blocks = num_blocks;
  p.q_rs = q_row_stride;
  p.q_hs = q_head_stride;
  p.k_bs = k_block_stride;
  p.k_ts = k_token_stride;
  p.k_hs = k_head_stride;
  p.v_bs = v_block_stride;
  p.v_ts = v_token_stride;
  p.v_hs = v_head_stride;
  p.t_rs = table_row_stride;
  p.scale_log2 = scale * 1.4426950408889634f;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool d128 = head_dim == 128;
  switch (dtype) {
    case RLT_BF16:
      return d128 ? launch<__nv_bfloat16, 128>(p, num_chunks, row_slots, suffix_lse, out, out_row_stride,
                                               out_head_stride, phases, s)
                  : launch<__nv_bfloat16, 64>(p, num_chunks, row_slots, suffix_lse, out, out_row_stride,
                                              out_head_stride, phases, s);
    case RLT_F16:
      return d128 ? launch<__half, 128>(p, num_chunks, row_slots, suffix_lse, out, out_row_stride,
                                        out_head_stride, phases, s)
                  : launch<__half, 64>(p, num_chunks, row_slots, suffix_lse, out, out_row_stride,
                                       out_head_stride, phases, s);
    default:
      return d128 ? launch<float, 128>(p, num_chunks, row_slots, suffix_lse, out, out_row_stride,
                                       out_head_stride, phases, s)
                  : launch<float, 64>(p, num_chunks, row_slots, suffix_lse, out, out_row_stride,
                                      out_head_stride, phases, s);
  }
}
}  // namespace

#define RLT_SHARED_ARGS                                                                       \
  q, key_cache, value_cache, block_tables, chunks, members, member_slots, row_slots,         \
      suffix_lse, out, workspace, workspace_size, status, dtype, num_rows, num_q_heads,      \
      num_kv_heads, head_dim, page_size, table_width, num_blocks, num_chunks, num_slots,     \
      num_members, q_row_stride, q_head_stride, k_block_stride, k_token_stride,             \
      k_head_stride, v_block_stride, v_token_stride, v_head_stride, table_row_stride,       \
      out_row_stride, out_head_stride, scale
#define RLT_SHARED_PARAMS                                                                     \
  const void *q, const void *key_cache, const void *value_cache,                             \
      const int32_t *block_tables, const int32_t *chunks, const int32_t *members,            \
      const int32_t *member_slots, const int32_t *row_slots, const float *suffix_lse,        \
      void *out, void *workspace, size_t workspace_size, int32_t *status, int32_t dtype,     \
      int32_t num_rows, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,         \
      int32_t page_size, int32_t table_width, int64_t num_blocks, int32_t num_chunks,        \
      int32_t num_slots, int32_t num_members, int64_t q_row_stride, int64_t q_head_stride,   \
      int64_t k_block_stride, int64_t k_token_stride, int64_t k_head_stride,                 \
      int64_t v_block_stride, int64_t v_token_stride, int64_t v_head_stride,                 \
      int64_t table_row_stride, int64_t out_row_stride, int64_t out_head_stride, float scale

extern "C" int rlt_paged_decode_shared(RLT_SHARED_PARAMS, void* stream) {
  return shared_entry(RLT_SHARED_ARGS, kPhaseChunks | kPhaseMerge, stream);
}

extern "C" int rlt_paged_decode_shared_phases(RLT_SHARED_PARAMS, int32_t phases, void* stream) {
  return shared_entry(RLT_SHARED_ARGS, phases, stream);
}
