// Paged decode attention that reads pages shared by several rows once.
//
// With prefix caching (vllm_rlt/core/kv_cache_manager.py:211-251: complete
// prompt pages are published by content hash and handed to later requests
// by reference, `_refs[b] += 1`), many rows of a decode batch point their
// tables at the same physical pages for a common prompt prefix. The plain
// decode kernel reads those pages once per row. Here a host-built plan cuts
// the work into chunks: a chunk is a token range of one table row together
// with the rows (members) that share it. One CTA per (chunk, KV head) reads
// each sub-tile of its chunk once (64 tokens on the 16-bit tensor-core path,
// 32 in fp32) and runs the online softmax of every (member row, query head)
// pair of its KV head on it, writing an fp32 partial (o, max, sum) per pair.
// Each row's own tokens after the shared prefix go through the plain decode
// kernel (rlt_paged_decode_lse on per-row suffix tables, on the caller's
// stream beside the chunks), which leaves the suffix result in `out` and its
// log-sum-exp in `suffix_lse`; a merge kernel then folds the prefix partials
// into `out`. Result = softmax(q K^T * scale) V over
// the row's context, the semantics of torch_paged_attention
// (vllm_rlt/kernels/paged_attention.py:12-36).
//
// Plan arrays (device int32): chunks[c] = {table_row, token_begin, token_end,
// member_begin, member_count}; members[member_begin + i] = row id;
// member_slots[...] = the partial slot of that (row, chunk); row_slots[r] ..
// row_slots[r+1] = the slots of row r. member_count * (Hq / Hkv) <= 32.
#include <atomic>
#include <type_traits>

#include "common.cuh"
#include "tc_ptx.cuh"

namespace rlt {
namespace {

constexpr int kSubTile = 32;   // tokens per shared-memory sub-tile (one per lane)
constexpr int kMaxPairs = 32;  // (member, query head) pairs per CTA
constexpr int kWarps = 4;
constexpr int kPairsPerWarp = kMaxPairs / kWarps;
constexpr int kPhaseChunks = 1;  // the prefix-chunk partials
constexpr int kPhaseMerge = 2;   // their merge into the suffix result

struct SharedParams {
  CUtensorMap kmap;  // kTma chunk kernel: {D, Hkv, page, blocks}, box {64, 1, page, 1}
  CUtensorMap vmap;
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
// TMA staging (kTma chunk kernel): per stage K then V, each [halves of 64
// dims][64 tokens][128 B] with the 128-byte swizzle (1024-byte aligned);
// the Q tile (padded rows, as above) and the stage barriers follow.
template <int D>
struct LayoutTma {
  static constexpr int kTokens = 64;
  // two stages: the next sub-tile lands while one is consumed. Three (108 KB
  // per CTA) were faster alone but left no room on an SM for the suffix
  // decode that runs beside this kernel (the call measured 314-340 us
  // against 253 us with two)
  static constexpr int kStages = 2;
  static constexpr int kHalves = D / 64;
  static constexpr int kHalfBytes = kTokens * 128;         // 64 tokens x 64 dims x 2 B
  static constexpr int kTileBytes = kHalves * kHalfBytes;  // one K or V sub-tile
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int kQOffset = kStages * kStageBytes;
  static constexpr int kBarOffset = kQOffset + (LayoutMma<D>::kQBytes + 1023) / 1024 * 1024;
  static constexpr int kBytes = kBarOffset + kStages * 8 + 1024;  // + alignment slack
  static constexpr int kCombineBytes = kWarps * 16 * (D + 2) * 4;
  static_assert(D % 64 == 0, "64-dim halves");
  static_assert(kCombineBytes <= kStages * kStageBytes, "merge buffer exceeds the K/V staging");
  static_assert(2 * (kBytes + 1024) <= 228 * 1024, "two CTAs per SM");
};
// Bound on a stage wait (cycles, ~50 ms at 1.9 GHz): a load that never lands
// ends the CTA with RLT_STATUS_TIMEOUT instead of a hang.
constexpr long long kTmaWaitLimit = 100000000LL;

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

// 1024-byte aligned start inside the dynamic shared memory (the 128-byte
// swizzle of a TMA load is a function of the shared-memory address).
__device__ __forceinline__ uint8_t* align1024(uint8_t* base) {
  return base + ((1024u - (smem_addr(base) & 1023u)) & 1023u);
}

// kTma = false: every thread copies its share of each 64-token sub-tile with
// cp.async from the page table (any page size). kTma = true (pages of 8, 16,
// 32 or 64 tokens): warp 0's lanes issue one tiled TMA load per page and
// 64-dim half of K and of V into 128-byte-swizzled stages (double buffered,
// bounded mbarrier waits), so no thread spends instructions on copies. The
// math is the same in both.
template <typename T, int D, bool kTma>
__global__ void __launch_bounds__(kWarps * 32, 2)
    shared_range_mma_kernel(const __grid_constant__ SharedParams p) {
  using L = LayoutMma<D>;
  using LT = LayoutTma<D>;
  constexpr int kKSteps = D / 16;  // k16 steps over the head dim (S = Q K^T)
  constexpr int kDTiles = D / 8;   // n8 tiles over the head dim (O)
  constexpr int kRowVecs = D / 8;  // 16-byte vectors per row
  constexpr int kTokens = L::kTokens;
  static_assert(LT::kTokens == kTokens, "one sub-tile size");
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = kTma ? align1024(smem_raw) : smem_raw;
  uint8_t* sq = kTma ? smem + LT::kQOffset : smem;
  uint8_t* skv = kTma ? smem : smem + L::kQBytes;  // K/V staging; later the slice merge
  uint64_t* bar_full = reinterpret_cast<uint64_t*>(smem + LT::kBarOffset);  // kTma only

  const int* c = p.chunks + blockIdx.x * 5;
  const int table_row = c[0], tok_begin = c[1], tok_end = c[2];
  const int member_begin = c[3], member_count = c[4];
  const int kvh = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pairs = member_count * p.group;
  if (pairs <= 0 || pairs > kMaxPairs || tok_begin < 0 || tok_begin >= tok_end ||
      table_row < 0 || table_row >= p.num_rows || member_begin < 0 ||
      member_begin + member_count > p.num_members) {
    if (tid == 0 && pairs != 0) raise_status(p.status, kStatusBadSequence);
    return;
  }
  const int tiles = pairs <= 16 ? 1 : 2;
  const int slices = kWarps / tiles;  // 4 or 2 token slices per sub-tile
  const int mt = warp % tiles, sl = warp / tiles;
  const int slice_tokens = kTokens / slices;  // 16 or 32
  const int g = lane >> 2, tig = lane & 3;
  const int64_t trow = static_cast<int64_t>(table_row) * p.t_rs;
  const T* kbase = static_cast<const T*>(p.k) + kvh * p.k_hs;
  const T* vbase = static_cast<const T*>(p.v) + kvh * p.v_hs;

  // ---- TMA staging: sub-tile u covers tokens t_first + 64 u ..; page j of
  // it goes to rows [j * page, (j + 1) * page) of every half of the stage.
  const int t_first = tok_begin - tok_begin % p.page;  // page-aligned start (kTma)
  const int n_tiles = (tok_end - t_first + kTokens - 1) / kTokens;
  const int ppt = kTokens / p.page;  // pages per sub-tile (kTma)
  // block coordinate of page j of sub-tile u; out of range (zero fill, no
  // DRAM read) past the chunk or for a bad id
  auto page_block = [&](int u, int j) {
    int blk = static_cast<int>(p.num_blocks);
    const int pos = t_first + u * kTokens + j * p.page;
    if (pos < tok_end) {
      const int pg = pos / p.page;
      if (pg >= p.width) {
        raise_status(p.status, kStatusBadLength);
      } else {
        const int b = p.tables[trow + pg];
        if (b >= 0 && b < p.num_blocks)
          blk = b;
        else
          raise_status(p.status, kStatusBadBlock);
      }
    }
    return blk;
  };
  int next_blk = 0;  // warp 0, lane j < ppt: page j of the next sub-tile to issue, read ahead
  auto issue = [&](int u) {  // warp 0
    const int st = u % LT::kStages;
    if (lane == 0) tc::mbar_expect_tx(&bar_full[st], LT::kStageBytes);
    __syncwarp();
    if (lane < ppt) {
      uint8_t* kd = skv + st * LT::kStageBytes + lane * p.page * 128;
      uint8_t* vd = kd + LT::kTileBytes;
#pragma unroll
      for (int h = 0; h < LT::kHalves; ++h) {
        tc::tma_load_4d(kd + h * LT::kHalfBytes, &p.kmap, &bar_full[st], h * 64, kvh, 0, next_blk);
        tc::tma_load_4d(vd + h * LT::kHalfBytes, &p.vmap, &bar_full[st], h * 64, kvh, 0, next_blk);
      }
      next_blk = page_block(u + 1, lane);
    }
  };
  if constexpr (kTma) {
    if (tid == 0) {
      for (int i = 0; i < LT::kStages; ++i) tc::mbar_init(&bar_full[i], 1);
      tc::fence_mbar_init();
    }
    __syncthreads();
    if (warp == 0) {
      if (lane == 0) {
        tc::prefetch_tensormap(&p.kmap);
        tc::prefetch_tensormap(&p.vmap);
      }
      if (lane < ppt) next_blk = page_block(0, lane);
      for (int u = 0; u < LT::kStages - 1 && u < n_tiles; ++u) issue(u);
    }
  }

  // Q of every pair, in the input type (rows >= pairs stay zero); 16-byte
  // loads when every row and head starts on a 16-byte boundary
  const bool q_vec = (reinterpret_cast<uintptr_t>(p.q) & 15) == 0 && p.q_rs % 8 == 0 &&
                     p.q_hs % 8 == 0;
  for (int e = tid; e < kMaxPairs * kRowVecs; e += kWarps * 32) {
    const int row = e / kRowVecs, v = e % kRowVecs;
    uint4 w = make_uint4(0, 0, 0, 0);
    if (row < pairs) {
      const int r = p.members[member_begin + row / p.group];
      const int qh = kvh * p.group + row % p.group;
      if (r >= 0 && r < p.num_rows) {
        const T* src = static_cast<const T*>(p.q) + r * p.q_rs + qh * p.q_hs + v * 8;
        if (q_vec) {
          w = *reinterpret_cast<const uint4*>(src);
        } else {
          uint32_t x[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            T two[2] = {src[2 * i], src[2 * i + 1]};
            x[i] = *reinterpret_cast<uint32_t*>(two);
          }
          w = make_uint4(x[0], x[1], x[2], x[3]);
        }
      }
    }
    *reinterpret_cast<uint4*>(sq + row * L::kRowBytes + v * 16) = w;
  }

  // ---- cp.async staging: 4 threads per token copy its K row and its V row,
  // each thread a quarter of both (vector j * 4 + quarter, so the 4 threads
  // of a token read 64 contiguous bytes per copy); a pass of the CTA covers
  // kPassTokens tokens. A thread keeps the page index and in-page offset of
  // each of its tokens and steps them by one sub-tile per call, so a copy
  // costs no division: per token one address, then 2 x kVecs copies. The
  // page ids a sub-tile's copies need are read when the previous sub-tile's
  // copies are issued, so the table's round trip never sits between a warp
  // and its math.
  auto tile_ptr = [&](int buf, int which) { return skv + (buf * 2 + which) * L::kTileBytes; };
  constexpr int kThreads = kWarps * 32;
  constexpr int kQuarter = 4;
  constexpr int kVecs = kRowVecs / kQuarter;  // 16-byte vectors per thread per row
  constexpr int kPassTokens = kThreads / kQuarter;
  constexpr int kPasses = kTokens / kPassTokens;
  static_assert(kRowVecs % kQuarter == 0 && kTokens % kPassTokens == 0, "loader mapping");
  const int quarter = tid % kQuarter, ltok = tid / kQuarter;
  const int step_pages = kTokens / p.page, step_off = kTokens % p.page;
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
    read_ids(t0 + kTokens);
  };
  if constexpr (!kTma) {
    read_ids(tok_begin);
    load_tile(0, tok_begin);
  }
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

  // shared-memory address of 16-byte chunk cf (over the head dim) of token row tok
  auto kv_addr = [&](const uint8_t* tile, int tok, int cf) -> uint32_t {
    if constexpr (kTma)
      return smem_addr(tile) + (cf >> 3) * LT::kHalfBytes + (tok >> 3) * 1024 + (tok & 7) * 128 +
             (((cf & 7) ^ (tok & 7)) << 4);
    else
      return smem_addr(tile + tok * L::kRowBytes + cf * 16);
  };

  // one staged sub-tile whose token 0 is t0
  auto consume = [&](const uint8_t* ktile, const uint8_t* vtile, int t0) {
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
          uint32_t b0, b1, b2, b3;
          ldsm_x4(kv_addr(ktile, tok0 + (j + (jj >> 1)) * 8 + r, ks * 2 + (jj & 1)), b0, b1, b2,
                  b3);
          mma16816<T>(s[j], qa[ks], b0, b1);
          mma16816<T>(s[j + 1], qa[ks], b2, b3);
        }
      }
    }
    // scale, mask the tokens outside the chunk, online softmax of rows g and g + 8
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (j * 8 >= slice_tokens) break;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tk = t0 + tok0 + j * 8 + 2 * tig + (e & 1);
        const bool inside = tk < tok_end && (!kTma || tk >= tok_begin);
        s[j][e] = inside ? s[j][e] * p.scale_log2 : -INFINITY;
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
        const int vtok = tok0 + kk * 16 + 8 * (jj & 1) + r;
#pragma unroll
        for (int n = 0; n < kDTiles; n += 2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(kv_addr(vtile, vtok, n + (jj >> 1)), b0, b1, b2, b3);
          mma16816<T>(o[n], a, b0, b1);
          mma16816<T>(o[n + 1], a, b2, b3);
        }
      }
    }
  };

  if constexpr (kTma) {
    for (int t = 0; t < n_tiles; ++t) {
      const int st = t % LT::kStages;
      const bool ok = tc::mbar_wait(&bar_full[st], (t / LT::kStages) & 1, kTmaWaitLimit);
      uint8_t* ktile = skv + st * LT::kStageBytes;
      uint8_t* vtile = ktile + LT::kTileBytes;
      const int t0 = t_first + t * kTokens;
      const int valid = tok_end - t0;
      if (ok && valid < kTokens) {
        // V rows past the chunk may hold any bits (NaN included) and P is 0
        // there: zero them so P V stays finite (the TMA writes have landed)
        for (int e = tid; e < (kTokens - valid) * LT::kHalves * 8; e += kWarps * 32) {
          const int tok = valid + e / (LT::kHalves * 8);
          const int h = (e / 8) % LT::kHalves, cidx = e % 8;
          *reinterpret_cast<uint4*>(vtile + h * LT::kHalfBytes + (tok >> 3) * 1024 +
                                    (tok & 7) * 128 + cidx * 16) = make_uint4(0, 0, 0, 0);
        }
      }
      // this sub-tile has landed everywhere, and every warp is done with the
      // stage the next load refills (it held sub-tile t - 1)
      if (__syncthreads_or(!ok)) {
        if (tid == 0) {
          raise_status(p.status, kStatusTimeout);
          // let the loads in flight land before the CTA's shared memory goes
          for (int u = t; u < n_tiles && u < t + LT::kStages - 1; ++u)
            tc::mbar_wait(&bar_full[u % LT::kStages], (u / LT::kStages) & 1, kTmaWaitLimit);
        }
        return;
      }
      if (warp == 0 && t + LT::kStages - 1 < n_tiles) issue(t + LT::kStages - 1);
      consume(ktile, vtile, t0);
    }
    __syncthreads();  // every warp is done with the last stage before the merge reuses it
  } else {
    int buf = 0;
    for (int t0 = tok_begin; t0 < tok_end; t0 += kTokens, buf ^= 1) {
      if (t0 + kTokens < tok_end) {
        load_tile(buf ^ 1, t0 + kTokens);
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncthreads();  // this sub-tile's K and V are in shared memory
      consume(tile_ptr(buf, 0), tile_ptr(buf, 1), t0);
      __syncthreads();  // every warp is done with this buffer before it is refilled
    }
  }

#pragma unroll
  for (int h = 0; h < 2; ++h) {
    lrow[h] += __shfl_xor_sync(kFullMask, lrow[h], 1);
    lrow[h] += __shfl_xor_sync(kFullMask, lrow[h], 2);
  }
  // merge the token slices of each M tile (the K/V staging is free now):
  // every warp stores its partial rows, then each warp merges a quarter of
  // the columns of every pair
  constexpr int kCbRow = D + 2;  // floats per staged row: o, then max and sum
  float* cb = reinterpret_cast<float*>(skv);
  {
    float* mine = cb + warp * 16 * kCbRow;
#pragma unroll
    for (int n = 0; n < kDTiles; ++n) {
      const int col = n * 8 + 2 * tig;
      *reinterpret_cast<float2*>(mine + g * kCbRow + col) = make_float2(o[n][0], o[n][1]);
      *reinterpret_cast<float2*>(mine + (g + 8) * kCbRow + col) = make_float2(o[n][2], o[n][3]);
    }
    if (tig == 0) {
      *reinterpret_cast<float2*>(mine + g * kCbRow + D) = make_float2(mrow[0], lrow[0]);
      *reinterpret_cast<float2*>(mine + (g + 8) * kCbRow + D) = make_float2(mrow[1], lrow[1]);
    }
  }
  __syncthreads();
  constexpr int kChunkCols = 8;                             // columns per work item
  constexpr int kItemsPerRow = D / kWarps / kChunkCols;     // items of one pair in one warp
  static_assert(D % (kWarps * kChunkCols) == 0, "epilogue column split");
  for (int it = lane; it < tiles * 16 * kItemsPerRow; it += 32) {
    const int pair = it / kItemsPerRow;  // = M tile * 16 + row
    const int col = (warp * kItemsPerRow + it % kItemsPerRow) * kChunkCols;
    if (pair >= pairs) continue;
    const int tile = pair / 16, row = pair % 16;
    float mxs = -INFINITY;
    for (int k = 0; k < slices; ++k)
      mxs = fmaxf(mxs, cb[((k * tiles + tile) * 16 + row) * kCbRow + D]);
    const float mref = mxs == -INFINITY ? 0.f : mxs;
    float acc[kChunkCols];
#pragma unroll
    for (int e = 0; e < kChunkCols; ++e) acc[e] = 0.f;
    float lsum = 0.f;
    for (int k = 0; k < slices; ++k) {
      const float* st = cb + ((k * tiles + tile) * 16 + row) * kCbRow;
      const float w = ex2(st[D] - mref);
      lsum += st[D + 1] * w;
#pragma unroll
      for (int e = 0; e < kChunkCols; e += 2) {
        const float2 x = *reinterpret_cast<const float2*>(st + col + e);
        acc[e] = fmaf(x.x, w, acc[e]);
        acc[e + 1] = fmaf(x.y, w, acc[e + 1]);
      }
    }
    const int slot = p.member_slots[member_begin + pair / p.group];
    if (slot < 0 || slot >= p.num_slots) {
      if (col == 0) raise_status(p.status, kStatusBadSequence);
      continue;
    }
    const int qh = kvh * p.group + pair % p.group;
    float4* dst = reinterpret_cast<float4*>(p.ws_o + (static_cast<int64_t>(slot) * p.hq + qh) * D + col);
#pragma unroll
    for (int e = 0; e < kChunkCols; e += 4)
      dst[e / 4] = make_float4(acc[e], acc[e + 1], acc[e + 2], acc[e + 3]);
    if (col == 0) {
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
int launch(const SharedParams& p, bool tma, int num_chunks, const int32_t* row_slots,
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
  } else if (tma) {
    constexpr int bytes = LayoutTma<D>::kBytes;
    static cudaError_t attr = cudaFuncSetAttribute(
        shared_range_mma_kernel<T, D, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (attr != cudaSuccess) return static_cast<int>(attr);
    if (num_chunks > 0)
      shared_range_mma_kernel<T, D, true>
          <<<dim3(num_chunks, p.hkv), kWarps * 32, bytes, stream>>>(p);
  } else {
    constexpr int bytes = LayoutMma<D>::kBytes;
    static cudaError_t attr = cudaFuncSetAttribute(
        shared_range_mma_kernel<T, D, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (attr != cudaSuccess) return static_cast<int>(attr);
    if (num_chunks > 0)
      shared_range_mma_kernel<T, D, false>
          <<<dim3(num_chunks, p.hkv), kWarps * 32, bytes, stream>>>(p);
  }
  if ((phases & kPhaseMerge) && p.num_rows > 0)
    shared_merge_kernel<T, D><<<dim3(p.num_rows, ceil_div(p.hq, kWarps)), kWarps * 32, 0, stream>>>(
        p.ws_o, p.ws_ml, row_slots, suffix_lse, out, p.hq, p.num_slots, o_rs, o_hs);
  return launch_status(cudaGetLastError());
}

// 2 (default): 16-bit chunks are staged by TMA where the page allows it; 1:
// always by cp.async. On the configs[1] prefix-cached batch the overlapped
// call took 253 us with TMA staging against 260 us with cp.async (4096-token
// chunks; 276 against 284 us with 512-token chunks): the TMA loader spends
// no instructions per copy.
std::atomic<int> g_shared_staging{2};

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace
}  // namespace rlt

namespace rlt {
namespace detail {
bool encode_kv_page_map(CUtensorMap* map, int32_t dtype, const void* base, int32_t head_dim,
                        int32_t hkv, int32_t page, int64_t num_blocks, int64_t bs, int64_t ts,
                        int64_t hs);
}  // namespace detail
}  // namespace rlt

using namespace rlt;

extern "C" int rlt_shared_prefix_select(int32_t staging) {
  if (staging != 1 && staging != 2) return g_shared_staging.load();
  return g_shared_staging.exchange(staging);
}

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
  // TMA staging: whole pages of 8..64 tokens tile a 64-token sub-tile, each
  // page's box lands 1024-byte aligned in the swizzled stage
  bool tma = false;
  if (dtype != RLT_F32 && (phases & kPhaseChunks) && num_chunks > 0 &&
      g_shared_staging.load() == 2 &&
      (page_size == 8 || page_size == 16 || page_size == 32 || page_size == 64) &&
      num_blocks > 0 && num_blocks < INT32_MAX)
    tma = detail::encode_kv_page_map(&p.kmap, dtype, key_cache, head_dim, num_kv_heads,
                                     page_size, num_blocks, k_block_stride, k_token_stride,
                                     k_head_stride) &&
          detail::encode_kv_page_map(&p.vmap, dtype, value_cache, head_dim, num_kv_heads,
                                     page_size, num_blocks, v_block_stride, v_token_stride,
                                     v_head_stride);
  const bool d128 = head_dim == 128;
  switch (dtype) {
    case RLT_BF16:
      return d128 ? launch<__nv_bfloat16, 128>(p, tma, num_chunks, row_slots, suffix_lse, out,
                                               out_row_stride, out_head_stride, phases, s)
                  : launch<__nv_bfloat16, 64>(p, tma, num_chunks, row_slots, suffix_lse, out,
                                              out_row_stride, out_head_stride, phases, s);
    case RLT_F16:
      return d128 ? launch<__half, 128>(p, tma, num_chunks, row_slots, suffix_lse, out,
                                        out_row_stride, out_head_stride, phases, s)
                  : launch<__half, 64>(p, tma, num_chunks, row_slots, suffix_lse, out,
                                       out_row_stride, out_head_stride, phases, s);
    default:
      return d128 ? launch<float, 128>(p, false, num_chunks, row_slots, suffix_lse, out,
                                       out_row_stride, out_head_stride, phases, s)
                  : launch<float, 64>(p, false, num_chunks, row_slots, suffix_lse, out,
                                      out_row_stride, out_head_stride, phases, s);
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
