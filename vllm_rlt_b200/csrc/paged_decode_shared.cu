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

// 16-bit K/V: the warps of a CTA split the chunk's (member, head) pairs into
// blocks of up to 8 and, when there are few pairs, split its 32-token
// sub-tiles between them (token splits are merged through shared memory at
// the end). Each lane holds its own token's K row in registers (loaded once
// per sub-tile, for all of the warp's pairs) and stages its V row into the
// warp's shared-memory slab; the probability-weighted V sum reads that slab.
template <int D>
struct Layout16 {
  static constexpr int kQFloats = kMaxPairs * D;          // pre-scaled q, fp32
  static constexpr int kSlabElems = kSubTile * D;         // one warp's V sub-tile
  static constexpr int kBytes = kQFloats * 4 + kWarps * kSlabElems * 2;
  // Token-split merge, reusing the same memory: with 4 splits a chunk has at
  // most 8 pairs, with 2 splits at most 16; entries [split][pair < 16] of
  // D + 2 floats (o, max, sum).
  static constexpr int kCombinePairs = 16;
  static constexpr int kCombineBytes = kWarps * kCombinePairs * (D + 2) * 4;
  static_assert(kCombineBytes <= kBytes, "token-split merge buffer exceeds shared memory");
};

template <typename T, int D>
__global__ void __launch_bounds__(kWarps * 32, 2) shared_range_kernel16(const SharedParams p) {
  constexpr int kE = D / 32;              // output dims per lane
  constexpr int kRowVecs = D / 8;         // 16-byte vectors per K/V row
  constexpr int kPW = 8;                  // pairs per warp
  extern __shared__ float4 smem4[];
  float* sq = reinterpret_cast<float*>(smem4);
  T* slab_all = reinterpret_cast<T*>(sq + Layout16<D>::kQFloats);

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
  const int blocks = pairs <= kPW ? 1 : pairs <= 2 * kPW ? 2 : 4;  // pair blocks
  const int splits = kWarps / blocks;                               // token splits
  const int pb = warp % blocks, ts = warp / blocks;
  const int pair0 = pb * kPW;
  const int npairs = min(kPW, pairs - pair0);

  for (int e = tid; e < pairs * D; e += kWarps * 32) {
    const int pair = e / D, d = e % D;
    const int row = p.members[member_begin + pair / p.group];
    const int qh = kvh * p.group + pair % p.group;
    float x = 0.f;
    if (row >= 0 && row < p.num_rows)
      x = to_f32<T>(static_cast<const T*>(p.q)[row * p.q_rs + qh * p.q_hs + d]);
    sq[e] = x * p.scale_log2;
  }
  __syncthreads();

  float m[kPW], l[kPW], o[kPW][kE];
#pragma unroll
  for (int i = 0; i < kPW; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int e = 0; e < kE; ++e) o[i][e] = 0.f;
  }
  T* slab = slab_all + warp * Layout16<D>::kSlabElems;
  const T* kbase = static_cast<const T*>(p.k) + kvh * p.k_hs;
  const T* vbase = static_cast<const T*>(p.v) + kvh * p.v_hs;

  for (int t0 = tok_begin + ts * kSubTile; t0 < tok_end; t0 += splits * kSubTile) {
    const int valid = min(kSubTile, tok_end - t0);
    uint4 kreg[kRowVecs];
#pragma unroll
    for (int v = 0; v < kRowVecs; ++v) kreg[v] = make_uint4(0, 0, 0, 0);
    if (lane < valid) {
      const int pos = t0 + lane;
      const int pg = pos / p.page;
      int b = -1;
      if (pg < p.width) {
        b = p.tables[table_row * p.t_rs + pg];
        if (b < 0 || b >= p.num_blocks) {
          raise_status(p.status, kStatusBadBlock);
          b = -1;
        }
      } else {
        raise_status(p.status, kStatusBadLength);
      }
      uint4* srow = reinterpret_cast<uint4*>(slab + lane * D);
      if (b >= 0) {
        const T* kr = kbase + b * p.k_bs + (pos % p.page) * p.k_ts;
        const T* vr = vbase + b * p.v_bs + (pos % p.page) * p.v_ts;
#pragma unroll
        for (int v = 0; v < kRowVecs; ++v) kreg[v] = ld_stream(kr + v * 8);
#pragma unroll
        for (int v = 0; v < kRowVecs; ++v) srow[v] = ld_stream(vr + v * 8);
      } else {
#pragma unroll
        for (int v = 0; v < kRowVecs; ++v) srow[v] = make_uint4(0, 0, 0, 0);
      }
    }
    __syncwarp();

#pragma unroll
    for (int i = 0; i < kPW; ++i) {
      if (i >= npairs) break;  // warp-uniform
      const float* qv = sq + (pair0 + i) * D;
      float s = 0.f;
#pragma unroll
      for (int v = 0; v < kRowVecs; ++v) {
        float kf[8];
        unpack16<T>(kreg[v], kf);
        const float4 a = *reinterpret_cast<const float4*>(qv + v * 8);
        const float4 b = *reinterpret_cast<const float4*>(qv + v * 8 + 4);
        s = fmaf(a.x, kf[0], s);
        s = fmaf(a.y, kf[1], s);
        s = fmaf(a.z, kf[2], s);
        s = fmaf(a.w, kf[3], s);
        s = fmaf(b.x, kf[4], s);
        s = fmaf(b.y, kf[5], s);
        s = fmaf(b.z, kf[6], s);
        s = fmaf(b.w, kf[7], s);
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
        const T* vr = slab + t * D + lane * kE;
        if constexpr (kE == 4) {
          const uint2 raw = *reinterpret_cast<const uint2*>(vr);
          float v0, v1, v2, v3;
          if constexpr (std::is_same<T, __nv_bfloat16>::value) {
            bf16x2_to_f32(raw.x, v0, v1);
            bf16x2_to_f32(raw.y, v2, v3);
          } else {
            f16x2_to_f32(raw.x, v0, v1);
            f16x2_to_f32(raw.y, v2, v3);
          }
          o[i][0] = fmaf(pt, v0, o[i][0]);
          o[i][1] = fmaf(pt, v1, o[i][1]);
          o[i][2] = fmaf(pt, v2, o[i][2]);
          o[i][3] = fmaf(pt, v3, o[i][3]);
        } else {
#pragma unroll
          for (int e = 0; e < kE; ++e) o[i][e] = fmaf(pt, to_f32<T>(vr[e]), o[i][e]);
        }
      }
    }
    __syncwarp();  // the slab is rewritten by the next sub-tile
  }

  // merge the token splits (shared memory reused: q and slabs are done)
  __syncthreads();
  float* cb = sq;  // [split][pair < kCombinePairs][D + 2]
  if (splits > 1) {
#pragma unroll
    for (int i = 0; i < kPW; ++i) {
      if (i >= npairs) break;
      float* st = cb + (ts * Layout16<D>::kCombinePairs + pair0 + i) * (D + 2);
#pragma unroll
      for (int e = 0; e < kE; ++e) st[lane * kE + e] = o[i][e];
      if (lane == 0) {
        st[D] = m[i];
        st[D + 1] = l[i];
      }
    }
    __syncthreads();
    if (ts != 0) return;
#pragma unroll
    for (int i = 0; i < kPW; ++i) {
      if (i >= npairs) break;
      float mx = -INFINITY;
      for (int k = 0; k < splits; ++k)
        mx = fmaxf(mx, cb[(k * Layout16<D>::kCombinePairs + pair0 + i) * (D + 2) + D]);
      float ls = 0.f, acc[kE] = {};
      for (int k = 0; k < splits; ++k) {
        const float* st = cb + (k * Layout16<D>::kCombinePairs + pair0 + i) * (D + 2);
        if (st[D + 1] <= 0.f) continue;
        const float w = ex2(st[D] - mx);
        ls += st[D + 1] * w;
#pragma unroll
        for (int e = 0; e < kE; ++e) acc[e] = fmaf(st[lane * kE + e], w, acc[e]);
      }
      m[i] = mx;
      l[i] = ls;
#pragma unroll
      for (int e = 0; e < kE; ++e) o[i][e] = acc[e];
    }
  }

#pragma unroll
  for (int i = 0; i < kPW; ++i) {
    if (i >= npairs) break;
    const int pair = pair0 + i;
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

size_t workspace_bytes(int64_t slots, int hq, int d) {
  return static_cast<size_t>(slots) * hq * (d + 2) * sizeof(float);
}

template <typename T, int D>
int launch(const SharedParams& p, int num_chunks, const int32_t* row_slots,
           const float* suffix_lse, void* out, int64_t o_rs, int64_t o_hs, cudaStream_t stream) {
  if constexpr (std::is_same<T, float>::value) {
    constexpr int bytes = SharedLayout<D>::kBytes;
    static cudaError_t attr = cudaFuncSetAttribute(
        shared_range_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (attr != cudaSuccess) return static_cast<int>(attr);
    if (num_chunks > 0)
      shared_range_kernel<T, D><<<dim3(num_chunks, p.hkv), kWarps * 32, bytes, stream>>>(p);
  } else {
    constexpr int bytes = Layout16<D>::kBytes;
    static cudaError_t attr = cudaFuncSetAttribute(
        shared_range_kernel16<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (attr != cudaSuccess) return static_cast<int>(attr);
    if (num_chunks > 0)
      shared_range_kernel16<T, D><<<dim3(num_chunks, p.hkv), kWarps * 32, bytes, stream>>>(p);
  }
  if (p.num_rows > 0)
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

extern "C" int rlt_paged_decode_shared(
    const void* q, const void* key_cache, const void* value_cache, const int32_t* block_tables,
    const int32_t* chunks, const int32_t* members, const int32_t* member_slots,
    const int32_t* row_slots, const float* suffix_lse, void* out, void* workspace,
    size_t workspace_size, int32_t* status,
    int32_t dtype, int32_t num_rows, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
    int32_t page_size, int32_t table_width, int64_t num_blocks, int32_t num_chunks,
    int32_t num_slots, int32_t num_members, int64_t q_row_stride, int64_t q_head_stride, int64_t k_block_stride,
    int64_t k_token_stride, int64_t k_head_stride, int64_t v_block_stride, int64_t v_token_stride,
    int64_t v_head_stride, int64_t table_row_stride, int64_t out_row_stride,
    int64_t out_head_stride, float scale, void* stream) {
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
  if (suffix_lse == nullptr && num_rows > 0) return RLT_E_SHAPE;
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
                                               out_head_stride, s)
                  : launch<__nv_bfloat16, 64>(p, num_chunks, row_slots, suffix_lse, out, out_row_stride,
                                              out_head_stride, s);
    case RLT_F16:
      return d128 ? launch<__half, 128>(p, num_chunks, row_slots, suffix_lse, out, out_row_stride,
                                        out_head_stride, s)
                  : launch<__half, 64>(p, num_chunks, row_slots, suffix_lse, out, out_row_stride,
                                       out_head_stride, s);
    default:
      return d128 ? launch<float, 128>(p, num_chunks, row_slots, suffix_lse, out, out_row_stride,
                                       out_head_stride, s)
                  : launch<float, 64>(p, num_chunks, row_slots, suffix_lse, out, out_row_stride,
                                      out_head_stride, s);
  }
}
