// Packed chunked-prefill paged causal attention on the sm_100a tensor cores.
//
// Semantics (vllm_rlt/kernels/flash_attention.py:66-96, FA4 varlen with a
// page table, causal, bottom-right aligned): sequence s owns query tokens
// cu[s] .. cu[s+1]-1 and keys 0 .. len_s-1 through its block table; query i
// of the chunk (0-based) sees keys 0 .. len_s - qlen_s + i.
//
// One CTA = (128-query tile of one sequence, one query head), 4 warps:
//  * TMA (tiled, never multicast) brings the Q tile and, per 128-key tile,
//    each K/V page of the head (a 4-D tensor map over the strided layer view
//    [blocks, page, Hkv, D]) into 128-byte-swizzled shared memory; pages past
//    the context or with a bad id are fetched at an out-of-range coordinate,
//    which the TMA unit fills with zeros;
//  * thread 0 issues tcgen05.mma: S = Q K^T (M=128, N=128, K=128) into TMEM
//    columns [0,128), then O += P V into TMEM columns [128,256);
//  * each thread owns one query row: it reads its S row with tcgen05.ld,
//    applies the causal mask and the scale, keeps a base-2 running max that
//    is only moved (and O rescaled in TMEM) when it grows by more than 2^8,
//    and writes P (input dtype) into swizzled shared memory for the PV MMA;
//  * K/V are double-buffered; every mbarrier wait is bounded and reports
//    RLT_STATUS_TIMEOUT instead of hanging.
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "tc_ptx.cuh"

namespace rlt {
namespace {

constexpr int kTileM = 128;
constexpr int kTileN = 128;
constexpr int kHeadDim = 128;
constexpr int kThreads = 128;
constexpr uint32_t kTmemCols = 256;       // S: [0, 128), O: [128, 256)
constexpr int kHalfBytes = 128 * 128;     // 128 rows x 64 columns x 2 B
constexpr int kTileBytes = 2 * kHalfBytes;
constexpr int kSmemBytes = 6 * kTileBytes + 1024;  // Q, K x2, V x2, P + alignment slack
constexpr long long kWaitLimit = 100000000LL;      // cycles (~50 ms at 1.9 GHz)
constexpr int32_t kStatusLayout = 64;  // dynamic shared memory base too far from 1024-byte alignment

struct PrefillTcParams {
  CUtensorMap qmap;  // {D, Hq, tokens}, box {64, 1, 128}
  CUtensorMap kmap;  // {D, Hkv, page, blocks}, box {64, 1, page, 1}
  CUtensorMap vmap;
  const int32_t* tables;
  const int32_t* lengths;
  const int32_t* cu;
  void* out;
  int32_t* status;
  int num_seqs, num_tokens, hq, group, page, width;
  int64_t num_blocks, t_rs, o_rs, o_hs;
  float scale_log2;
  // kSplitP kernels: a query tile whose first row attends fewer keys than
  // this splits P into hi + lo for every key tile (INT32_MAX: every tile)
  int split_keys;
};

// Byte offset of 16-byte chunk c of row r inside one [128 rows x 128 B]
// half-tile stored with the 128-byte swizzle (chunk index XOR row % 8).
__device__ __forceinline__ uint32_t sw128(int r, int c) {
  return static_cast<uint32_t>((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Key rows past the context in the last key tile. The tile is copied a whole
// page at a time, so the rows of the last context page beyond the context
// hold whatever the pool held there -- possibly NaN or Inf bit patterns in a
// pool allocated without initialisation. Their scores are masked (P = 0),
// but 0 x NaN is NaN in the PV product, so their V rows must be zeros. Rows
// of pages wholly past the context were zero-filled by the copy already.
// Called by one thread once the tile has landed; the caller then fences the
// generic writes against the tensor core's async-proxy reads.
__device__ __forceinline__ void zero_tail_rows(uint8_t* v_tile, int ctx, int tile_start, int page) {
  const int r0 = ctx - tile_start;
  const int page_end = (ctx + page - 1) / page * page;
  const int r1 = min(kTileN, page_end - tile_start);
  if (r0 < 0 || r0 >= r1) return;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  for (int r = r0; r < r1; ++r)  // a row is 128 contiguous bytes of each 64-column half
#pragma unroll
    for (int half = 0; half < 2; ++half)
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(v_tile + half * kHalfBytes + r * 128 + c * 16) = zero;
}

// The two 16-bit values of a pack2 word, widened exactly to fp32.
template <typename T>
__device__ __forceinline__ void unpack2(uint32_t w, float& lo, float& hi);
template <>
__device__ __forceinline__ void unpack2<__nv_bfloat16>(uint32_t w, float& lo, float& hi) {
  lo = __uint_as_float(w << 16);
  hi = __uint_as_float(w & 0xffff0000u);
}
template <>
__device__ __forceinline__ void unpack2<__half>(uint32_t w, float& lo, float& hi) {
  const __half2 v = *reinterpret_cast<const __half2*>(&w);
  lo = __low2float(v);
  hi = __high2float(v);
}


// ---- softmax arithmetic helpers (sm_100 packed fp32x2 and 3-input max) ----

__device__ __forceinline__ uint64_t pk2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void upk2(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// 2^x of a pair on the FMA pipe, to take part of the exponentials off the
// MUFU unit. x = n + f with n = rint(x) (adding and removing 1.5 * 2^23
// rounds to an integer), 2^f from a degree-3 polynomial fitted for this
// kernel (least-squares minimax of the relative error on [-0.5, 0.5]; largest
// relative error 7.5e-5 in fp32 Horner form, far below the bf16/fp16
// rounding of P), 2^n written into the exponent field. Arguments are clamped
// at -127, where that field is 0, so -inf gives 0 as ex2.approx.ftz does
// (results under 2^-126 may stay denormal where that flushes them).
__device__ __forceinline__ uint64_t exp2_poly2(float x0, float x1) {
  constexpr float kRound = 12582912.f;  // 1.5 * 2^23
  constexpr float kC0 = 0.9999281167984009f, kC1 = 0.6932609677314758f;
  constexpr float kC2 = 0.24261054396629333f, kC3 = 0.05517132207751274f;
  const uint64_t x = pk2(fmaxf(x0, -127.f), fmaxf(x1, -127.f));
  const uint64_t t = add2(x, pk2(kRound, kRound));
  const uint64_t n = add2(t, pk2(-kRound, -kRound));
  const uint64_t f = fma2(n, pk2(-1.f, -1.f), x);
  uint64_t q = fma2(pk2(kC3, kC3), f, pk2(kC2, kC2));
  q = fma2(q, f, pk2(kC1, kC1));
  q = fma2(q, f, pk2(kC0, kC0));
  float t0, t1;
  upk2(t, t0, t1);
  // the low bits of t hold 0x400000 + n: shifted into the exponent field
  // they give n (mod 2^32), to which the bias is added
  const uint32_t e0 = (static_cast<uint32_t>(__float_as_int(t0)) << 23) + 0x3F800000u;
  const uint32_t e1 = (static_cast<uint32_t>(__float_as_int(t1)) << 23) + 0x3F800000u;
  return mul2(q, pk2(__uint_as_float(e0), __uint_as_float(e1)));
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

template <typename T>
struct Fmt;
template <>
struct Fmt<__half> {
  static constexpr uint32_t value = 0;
};
template <>
struct Fmt<__nv_bfloat16> {
  static constexpr uint32_t value = 1;
};

// Warp 0: map blockIdx.x to (sequence, first query of the tile) by a running
// prefix over ceil(qlen_s / 128). Returns seq = -1 past the last tile.
template <int kRows = kTileM, bool kHeavyFirst = false>
__device__ void find_tile(const int32_t* cu, int num_seqs, int target, int lane, int* seq_out,
                          int* m0_out) {
  int running = 0;
  for (int base = 0; base < num_seqs; base += 32) {
    const int s = base + lane;
    int tiles = 0;
    if (s < num_seqs) {
      const int qlen = cu[s + 1] - cu[s];
      tiles = qlen > 0 ? (qlen + kRows - 1) / kRows : 0;
    }
    int incl = tiles;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(kFullMask, incl, o);
      if (lane >= o) incl += y;
    }
    const int excl = running + incl - tiles;
    const bool mine = s < num_seqs && target >= excl && target < excl + tiles;
    const unsigned hit = __ballot_sync(kFullMask, mine);
    if (mine) {
      *seq_out = s;
      // Later query tiles see more keys: with kHeavyFirst a sequence's last
      // tile is dispatched first, so long CTAs start early in the launch.
      const int idx = kHeavyFirst ? tiles - 1 - (target - excl) : target - excl;
      *m0_out = idx * kRows;
    }
    if (hit) return;
    running += __shfl_sync(kFullMask, incl, 31);
  }
  if (lane == 0) {
    *seq_out = -1;
    *m0_out = 0;
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    paged_prefill_tc_kernel(const __grid_constant__ PrefillTcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;
  uint8_t* sK[2] = {smem + kTileBytes, smem + 2 * kTileBytes};
  uint8_t* sV[2] = {smem + 3 * kTileBytes, smem + 4 * kTileBytes};
  uint8_t* sP = smem + 5 * kTileBytes;

  __shared__ __align__(8) uint64_t bar_q, bar_kv[2], bar_s, bar_pv;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int tile_seq, tile_m0, abort_flag;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int head = blockIdx.y;
  const int kvh = head / p.group;

  if (warp == 0) find_tile(p.cu, p.num_seqs, blockIdx.x, lane, &tile_seq, &tile_m0);
  if (tid == 0) {
    tc::mbar_init(&bar_q, 1);
    tc::mbar_init(&bar_kv[0], 1);
    tc::mbar_init(&bar_kv[1], 1);
    tc::mbar_init(&bar_s, 1);
    tc::mbar_init(&bar_pv, 1);
    tc::fence_mbar_init();
    abort_flag = 0;
  }
  __syncwarp();
  if (warp == 0) tc::tmem_alloc(&tmem_base_sh, kTmemCols);  // warp-collective
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  const uint32_t s_tmem = tmem;
  const uint32_t o_tmem = tmem + kTileN;
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;

  int seq = tile_seq;
  const int m0 = tile_m0;
  int qbegin = 0, qlen = 0, ctx = 0, n_tiles = 0;
  if (seq >= 0) {
    qbegin = p.cu[seq];
    qlen = p.cu[seq + 1] - qbegin;
    ctx = p.lengths[seq];
    if (qbegin < 0 || qlen <= 0 || qbegin + qlen > p.num_tokens || ctx < 0 ||
        static_cast<int64_t>(ctx) > static_cast<int64_t>(p.width) * p.page) {
      if (tid == 0) raise_status(p.status, kStatusBadSequence);
      seq = -1;
    } else {
      const int kmax = ctx - qlen + min(qlen - 1, m0 + kTileM - 1);
      n_tiles = kmax >= 0 ? kmax / kTileN + 1 : 0;
    }
  }

  const int pages_per_tile = kTileN / p.page;
  int issued = -1;  // last K/V tile whose loads thread 0 issued
  auto load_kv = [&](int t) {
    const int st = t & 1;
    tc::mbar_expect_tx(&bar_kv[st], 2 * kTileBytes);
    for (int pg = 0; pg < pages_per_tile; ++pg) {
      const int logical = t * pages_per_tile + pg;
      int blk = static_cast<int>(p.num_blocks);  // out of range: zero fill
      if (logical * p.page < ctx) {
        const int b = p.tables[seq * p.t_rs + logical];
        if (b >= 0 && b < p.num_blocks)
          blk = b;
        else
          raise_status(p.status, kStatusBadBlock);
      }
      const int row_off = pg * p.page * 128;
#pragma unroll
      for (int dh = 0; dh < 2; ++dh) {
        tc::tma_load_4d(sK[st] + dh * kHalfBytes + row_off, &p.kmap, &bar_kv[st], dh * 64, kvh,
                        0, blk);
        tc::tma_load_4d(sV[st] + dh * kHalfBytes + row_off, &p.vmap, &bar_kv[st], dh * 64, kvh,
                        0, blk);
      }
    }
    issued = t;
  };

  const int qi = m0 + tid;  // this thread's query row within the sequence chunk
  const int row_limit = min(ctx - qlen + qi, ctx - 1);
  float m_used = -INFINITY;
  float l_sum = 0.f;
  const uint32_t idesc_qk = tc::idesc_f16(Fmt<T>::value, kTileM, kTileN, 0);
  const uint32_t idesc_pv = tc::idesc_f16(Fmt<T>::value, kTileM, kHeadDim, 1);
  int done_tiles = 0;
  int s_commits = 0, pv_commits = 0;  // thread 0: commits issued on bar_s / bar_pv

  if (seq >= 0 && n_tiles > 0) {
    if (tid == 0) {
      tc::mbar_expect_tx(&bar_q, kTileBytes);
      tc::tma_load_3d(sQ, &p.qmap, &bar_q, 0, head, qbegin + m0);
      tc::tma_load_3d(sQ + kHalfBytes, &p.qmap, &bar_q, 64, head, qbegin + m0);
      load_kv(0);
      if (n_tiles > 1) load_kv(1);
      if (!tc::mbar_wait(&bar_q, 0, kWaitLimit)) abort_flag = 1;
    }
    for (int t = 0; t < n_tiles; ++t) {
      const int st = t & 1;
      if (tid == 0 && !abort_flag) {
        if (tc::mbar_wait(&bar_kv[st], (t >> 1) & 1, kWaitLimit)) {
          tc::tc_fence_after();
          if (t == n_tiles - 1) {
            zero_tail_rows(sV[st], ctx, t * kTileN, p.page);
            tc::fence_proxy_async_smem();
          }
#pragma unroll
          for (int ks = 0; ks < kHeadDim / 16; ++ks) {
            const uint32_t off = (ks >> 2) * kHalfBytes + (ks & 3) * 32;
            tc::mma_f16_ss(s_tmem, tc::smem_desc_sw128(tc::smem_u32(sQ) + off, 16, 1024),
                           tc::smem_desc_sw128(tc::smem_u32(sK[st]) + off, 16, 1024), idesc_qk,
                           ks > 0);
          }
          tc::mma_commit(&bar_s);
          ++s_commits;
        } else {
          abort_flag = 1;
        }
      }
      __syncthreads();
      if (abort_flag) break;
      if (!tc::mbar_wait(&bar_s, t & 1, kWaitLimit)) abort_flag = 1;
      tc::tc_fence_after();

      // ---- softmax on this thread's S row (128 keys)
      uint32_t sr[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tc::tmem_ld32(s_tmem + lane_base + c * 32, sr[c]);
#pragma unroll
      for (int c = 0; c < 4; ++c) tc::tmem_ld_wait(sr[c]);
      const int n0 = t * kTileN;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int key = n0 + c * 32 + j;
          const float s = key <= row_limit ? __uint_as_float(sr[c][j]) * p.scale_log2 : -INFINITY;
          sr[c][j] = __float_as_uint(s);
          mx = fmaxf(mx, s);
        }
      }
      const float m_new = fmaxf(m_used, mx);
      float factor = 1.f;
      if (m_new > m_used + 8.f) {  // includes the first finite max (m_used = -inf)
        factor = ex2(m_used - m_new);
        m_used = m_new;
      }
      const float mref = m_used == -INFINITY ? 0.f : m_used;
      uint32_t packed[64];
      float psum = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float p0 = ex2(__uint_as_float(sr[c][j]) - mref);
          const float p1 = ex2(__uint_as_float(sr[c][j + 1]) - mref);
          psum += p0 + p1;
          packed[c * 16 + j / 2] = pack2<T>(p0, p1);
        }
      }
      l_sum = l_sum * factor + psum;

      // PV of the previous tile must be done before P is overwritten and O
      // is rescaled; it also frees the K/V stage for tile t + 1.
      if (t > 0) {
        if (!tc::mbar_wait(&bar_pv, (t - 1) & 1, kWaitLimit)) abort_flag = 1;
        tc::tc_fence_after();
        if (tid == 0 && t + 1 < n_tiles && !abort_flag) load_kv(t + 1);
        // tcgen05.ld/st are warp-collective (.sync.aligned): the whole warp
        // rescales when any of its rows moved its max (factor is 1 elsewhere).
        if (__any_sync(kFullMask, factor != 1.f)) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tc::tmem_ld32(o_tmem + lane_base + c * 32, o);
            tc::tmem_ld_wait(o);
#pragma unroll
            for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * factor);
            tc::tmem_st32(o_tmem + lane_base + c * 32, o);
          }
          tc::tmem_st_wait();
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const int base = h * 32 + c * 4;
          *reinterpret_cast<uint4*>(sP + h * kHalfBytes + sw128(tid, c)) =
              make_uint4(packed[base], packed[base + 1], packed[base + 2], packed[base + 3]);
        }
      }
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      __syncthreads();
      if (abort_flag) break;
      if (tid == 0) {
        tc::tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < kTileN / 16; ++ks) {
          const uint32_t aoff = (ks >> 2) * kHalfBytes + (ks & 3) * 32;
          tc::mma_f16_ss(o_tmem, tc::smem_desc_sw128(tc::smem_u32(sP) + aoff, 16, 1024),
                         tc::smem_desc_sw128(tc::smem_u32(sV[st]) + ks * 2048, kHalfBytes, 1024),
                         idesc_pv, (t > 0 || ks > 0) ? 1u : 0u);
        }
        tc::mma_commit(&bar_pv);
        ++pv_commits;
      }
      done_tiles = t + 1;
    }
    if (done_tiles == n_tiles && !abort_flag) {
      if (!tc::mbar_wait(&bar_pv, (n_tiles - 1) & 1, kWaitLimit)) abort_flag = 1;
      tc::tc_fence_after();
    }
  }
  __syncthreads();
  if (abort_flag) {
    // Give in-flight copies and MMAs a bounded chance to land before the
    // shared memory and TMEM are released.
    if (tid == 0) {
      raise_status(p.status, kStatusTimeout);
      for (int t = done_tiles; t <= issued; ++t)
        tc::mbar_wait(&bar_kv[t & 1], (t >> 1) & 1, kWaitLimit);
      if (s_commits > 0) tc::mbar_wait(&bar_s, (s_commits - 1) & 1, kWaitLimit);
      if (pv_commits > 0) tc::mbar_wait(&bar_pv, (pv_commits - 1) & 1, kWaitLimit);
    }
  } else if (seq >= 0) {
    // seq and n_tiles are uniform over the CTA, so every warp reads its TMEM
    // lanes with all 32 threads; only rows inside the chunk are stored.
    const bool store = qi < qlen;
    T* dst = static_cast<T*>(p.out) + (qbegin + (store ? qi : 0)) * p.o_rs + head * p.o_hs;
    const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t o[32];
      if (n_tiles > 0) {
        tc::tmem_ld32(o_tmem + lane_base + c * 32, o);
        tc::tmem_ld_wait(o);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] = 0u;
      }
      if (!store) continue;
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        uint4 w;
        w.x = pack2<T>(__uint_as_float(o[v * 8 + 0]) * inv, __uint_as_float(o[v * 8 + 1]) * inv);
        w.y = pack2<T>(__uint_as_float(o[v * 8 + 2]) * inv, __uint_as_float(o[v * 8 + 3]) * inv);
        w.z = pack2<T>(__uint_as_float(o[v * 8 + 4]) * inv, __uint_as_float(o[v * 8 + 5]) * inv);
        w.w = pack2<T>(__uint_as_float(o[v * 8 + 6]) * inv, __uint_as_float(o[v * 8 + 7]) * inv);
        *reinterpret_cast<uint4*>(dst + c * 32 + v * 8) = w;
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}


// ---------------------------------------------------------------------------
// Warp-specialised version: one CTA = two 128-query tiles (A, B) of one
// sequence and head, 10 warps:
//   warps 0-3  softmax of tile A (one query row per thread, TMEM lanes 0-127)
//   warps 4-7  softmax of tile B
//   warp 8     issues the tcgen05.mma (one elected thread)
//   warp 9     issues the TMA loads (one elected thread)
// Variants: kHalves = 2 doubles the softmax warps (two per 32 rows, one per
// half of the key columns; MMA and producer become warps 16 and 17). kWide
// keeps one softmax warp per 32 rows, adds idle warps 10-11 and moves
// registers from warpgroup 2 to the softmax warpgroups so a row's 128 scores
// stay in registers between the row max and the exponentials.
// TMEM (512 columns): S_A [0,128), S_B [128,256), O_A [256,384), O_B [384,512).
// Shared memory: Q_A, Q_B, K, V, P_A, P_B (32 KiB each, 128-byte swizzle).
// Hand-offs are mbarriers only. The MMA issue order per key tile t is
//   PV_A(t), S_A(t+1), PV_B(t), S_B(t+1)
// so the softmax of one tile runs while the tensor core works on the other.
// K and V are single-buffered with separate release barriers: K(t+1) loads
// once both S(t) MMAs are done, V(t+1) once both PV(t) MMAs are done.

constexpr int kPairRows = 2 * kTileM;
constexpr uint32_t kPairTmemCols = 512;
// Threads of the two-tile kernel: 8 softmax warps per key-column half, the
// MMA warp and the producer warp; the wide-register variant adds two idle
// warps so that the MMA and producer warps form a whole warpgroup, which
// gives its registers to the softmax warpgroups (setmaxnreg acts per
// warpgroup).
constexpr int pair_threads(int halves, bool wide) { return wide ? 12 * 32 : (8 * halves + 2) * 32; }
// Register split of the wide variant: launched at 168 per thread (384
// threads), the softmax warpgroups rise to 200 and the MMA/producer
// warpgroup drops to 96: 256 x 200 + 128 x 96 = 63,488 <= 384 x 168 = 64,512.
// (216/64 and 208/80 fit as well but spill more in the MMA and producer code.)
constexpr int kWideLaunchRegs = 168;
// Of every 8 score pairs of a row, how many the wide softmax exponentiates
// with the FMA-pipe polynomial instead of the MUFU unit. 1, 2 and 3 each
// measured slower (4-8 %) on the prefill workload: the kernel runs at the
// power cap, so the extra instructions cost clock rather than freeing MUFU.
constexpr int kPolyPairs = 0;
constexpr int kWideSoftRegs = 200;
constexpr int kWideOtherRegs = 96;
static_assert(256 * kWideSoftRegs + 128 * kWideOtherRegs <= 384 * kWideLaunchRegs,
              "register split exceeds the launch allocation");

// The two softmax warps that share 32 query rows (kHalves = 2) meet at named
// barrier 1 + 4 x + quarter; the and-reduction carries a flag so that both
// leave the key loop together.
__device__ __forceinline__ bool pair_barrier_and(uint32_t id, bool pred) {
  uint32_t all;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\t"
      "setp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.and.pred po, %2, 64, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(all)
      : "r"(static_cast<uint32_t>(pred)), "r"(id)
      : "memory");
  return all != 0;
}

__device__ __forceinline__ void pair_barrier(uint32_t id) {
  asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory");
}
// K(t), V(t) stream through a ring of 32 KiB slots: item 2t = K(t), 2t+1 =
// V(t), slot = item % slots. With P in TMEM (kPTmem) the two P buffers of
// shared memory go to the ring instead: 5 slots rather than 3.
constexpr int kMaxRingSlots = 5;
// Barriers, flags and the softmax pair exchange, after the tiles in dynamic
// shared memory (the kernel has no static shared memory).
struct PairShared {
  uint64_t bar_q, bar_full[kMaxRingSlots], bar_empty[kMaxRingSlots];
  uint64_t bar_s[2], bar_p[2], bar_pv[2];
  uint32_t tmem_base;
  int tile_seq, tile_m0, abort_flag;
  float pair_red[2 * 2 * kTileM];  // row max, then row sum, per (tile, half, row)
};
constexpr int kMaxSmem = 227 * 1024;
template <bool kPTmem>
struct PairLayout {
  static constexpr int kSlots = kPTmem ? 5 : 3;
  static constexpr int kPBuffers = kPTmem ? 0 : 2;
  static constexpr int kTileRegion = (2 + kPBuffers + kSlots) * kTileBytes;
  // all a CTA may have: the tiles need a 1024-byte aligned start, and the
  // allocation's base is aligned at least that well in practice; the kernel
  // checks that the slack covers the distance it must skip
  static constexpr int kSmemBytes = kMaxSmem;
  static constexpr int kSlack = kSmemBytes - kTileRegion - static_cast<int>(sizeof(PairShared));
};
static_assert(PairLayout<true>::kSlack >= 0 && PairLayout<false>::kSlack >= 0,
              "shared memory per CTA");

// kSplitP (wide variant only): in a query tile that splits (its first row
// attends fewer than p.split_keys keys), P is handed to the PV product as
// two 16-bit operands, P_hi = round(P) in S_x's first 64 columns and P_lo =
// round(P - P_hi) in its last 64, and O_x accumulates P_hi V + P_lo V. P
// then carries about 16 significant bits instead of 8 (bf16), which takes
// the rounding of P out of the output's error where it matters: a row that
// attends few keys sees the bf16 rounding of each probability (up to 2^-9
// relative) almost unaveraged, while over hundreds of keys the independent
// roundings average out (relative error ~ 2^-9 / sqrt(keys)). The decision is
// per query tile and made identically by its softmax warps and the MMA
// thread from the tile's position, so both agree without a hand-off.
template <typename T, bool kPTmem, int kHalves, bool kWide, bool kSplitP>
__device__ __forceinline__ void pair_body(const PrefillTcParams& p) {
  static_assert(kHalves == 1 || (kHalves == 2 && kPTmem), "split softmax needs P in TMEM");
  static_assert(!kWide || (kHalves == 1 && kPTmem), "wide registers: one warp per row set");
  static_assert(!kSplitP || kWide, "the split P needs the register-resident scores");
  constexpr int kRingSlots = PairLayout<kPTmem>::kSlots;
  constexpr int kSoftWarps = 8 * kHalves;
  constexpr int kMmaWarp = kSoftWarps;
  constexpr int kProducerWarp = kSoftWarps + 1;
  constexpr int kCols = kTileN / kHalves;     // key columns of S per softmax warp
  constexpr int kOCols = kHeadDim / kHalves;  // O columns each softmax warp rescales and stores
  // declared without an alignment the compiler could fold the check below into
  extern __shared__ uint8_t smem_raw[];
  const uintptr_t raw = reinterpret_cast<uintptr_t>(smem_raw);
  const uintptr_t skip = ((raw + 1023) & ~static_cast<uintptr_t>(1023)) - raw;
  if (skip > static_cast<uintptr_t>(PairLayout<kPTmem>::kSlack)) {  // uniform: no access yet
    if (threadIdx.x == 0) raise_status(p.status, kStatusLayout);
    return;
  }
  uint8_t* smem = smem_raw + skip;
  uint8_t* sQ[2] = {smem, smem + kTileBytes};
  // P_x (shared-memory variant only) at smem + (2 + x) * kTileBytes
  uint8_t* ring = smem + (2 + PairLayout<kPTmem>::kPBuffers) * kTileBytes;
  PairShared& sh = *reinterpret_cast<PairShared*>(smem + PairLayout<kPTmem>::kTileRegion);
  uint64_t& bar_q = sh.bar_q;
  uint64_t* bar_full = sh.bar_full;
  uint64_t* bar_empty = sh.bar_empty;
  uint64_t* bar_s = sh.bar_s;
  uint64_t* bar_p = sh.bar_p;
  uint64_t* bar_pv = sh.bar_pv;
  uint32_t& tmem_base_sh = sh.tmem_base;
  int& tile_seq = sh.tile_seq;
  int& tile_m0 = sh.tile_m0;
  int& abort_flag = sh.abort_flag;
  float* pair_red = sh.pair_red;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int head = blockIdx.y;
  const int kvh = head / p.group;

  if (warp == 0)
    find_tile<kPairRows, true>(p.cu, p.num_seqs, blockIdx.x, lane, &tile_seq, &tile_m0);
  if (tid == 0) {
    tc::mbar_init(&bar_q, 1);
    for (int i = 0; i < kRingSlots; ++i) {
      tc::mbar_init(&bar_full[i], 1);
      tc::mbar_init(&bar_empty[i], 1);
    }
    for (int x = 0; x < 2; ++x) {
      tc::mbar_init(&bar_s[x], 1);
      tc::mbar_init(&bar_p[x], kSoftWarps / 2);  // one arrival per softmax warp
      tc::mbar_init(&bar_pv[x], 1);
    }
    tc::fence_mbar_init();
    abort_flag = 0;
  }
  __syncwarp();
  if (warp == 0) tc::tmem_alloc(&tmem_base_sh, kPairTmemCols);  // warp-collective
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  volatile int* aborted = &abort_flag;  // set by any role on a timed-out wait

  int seq = tile_seq;
  const int m0 = tile_m0;
  int qbegin = 0, qlen = 0, ctx = 0, n_tiles = 0;
  if (seq >= 0) {
    qbegin = p.cu[seq];
    qlen = p.cu[seq + 1] - qbegin;
    ctx = p.lengths[seq];
    if (qbegin < 0 || qlen <= 0 || qbegin + qlen > p.num_tokens || ctx < 0 ||
        static_cast<int64_t>(ctx) > static_cast<int64_t>(p.width) * p.page) {
      if (tid == 0) raise_status(p.status, kStatusBadSequence);
      seq = -1;
    } else {
      const int kmax = ctx - qlen + min(qlen - 1, m0 + kPairRows - 1);
      n_tiles = kmax >= 0 ? kmax / kTileN + 1 : 0;
    }
  }
  const bool active = seq >= 0 && n_tiles > 0;

  auto producer_role = [&]() {
    // ---------------- TMA producer. The warp's lanes fetch the block ids of
    // a key tile together (lane j: page j) a tile ahead of its copies and
    // check them only when the copies are issued, so neither the table read
    // nor its latency sits between two copies; lane j issues page j's copies.
    const int pages_per_tile = kTileN / p.page;
    struct PageId {
      int raw;
      bool live;  // a page of the context (else the copy zero-fills)
    };
    auto tile_pages = [&](int t) {
      PageId id{0, false};
      const int logical = t * pages_per_tile + lane;
      if (lane < pages_per_tile && t < n_tiles && logical * p.page < ctx) {
        id.raw = p.tables[seq * p.t_rs + logical];
        id.live = true;
      }
      return id;
    };
    auto block_of = [&](PageId id) {
      int blk = static_cast<int>(p.num_blocks);  // out of range: zero fill
      if (id.live) {
        if (id.raw >= 0 && id.raw < p.num_blocks)
          blk = id.raw;
        else
          raise_status(p.status, kStatusBadBlock);
      }
      return blk;
    };
    if (lane == 0) {
      tc::prefetch_tensormap(&p.qmap);
      tc::prefetch_tensormap(&p.kmap);
      tc::prefetch_tensormap(&p.vmap);
    }
    int cur = block_of(tile_pages(0));
    PageId nxt = tile_pages(1);
    if (lane == 0) {
      tc::mbar_expect_tx(&bar_q, 2 * kTileBytes);
      for (int x = 0; x < 2; ++x)
        for (int dh = 0; dh < 2; ++dh)
          tc::tma_load_3d(sQ[x] + dh * kHalfBytes, &p.qmap, &bar_q, dh * 64, head,
                          qbegin + m0 + x * kTileM);
    }
    // item i: K(i/2) when i is even, V(i/2) when odd; slot i % slots. A slot
    // is refilled once the MMA that last read its previous item committed
    // the slot's empty barrier.
    const int items = 2 * n_tiles;
    int issued = 0;
    bool stop = false;
    for (int i = 0; i < items; ++i) {
      const int slot = i % kRingSlots;
      int ok = 1;
      if (lane == 0)
        ok = *aborted == 0 &&
             (i < kRingSlots ||
              tc::mbar_wait(&bar_empty[slot], (i / kRingSlots - 1) & 1, kWaitLimit));
      if (!__shfl_sync(kFullMask, ok, 0)) {
        stop = true;
        break;
      }
      uint8_t* dst = ring + slot * kTileBytes;
      const CUtensorMap* map = (i & 1) ? &p.vmap : &p.kmap;
      if (lane == 0) tc::mbar_expect_tx(&bar_full[slot], kTileBytes);
      __syncwarp();
      if (lane < pages_per_tile) {  // lane j copies page j of the tile
#pragma unroll
        for (int dh = 0; dh < 2; ++dh)
          tc::tma_load_4d(dst + dh * kHalfBytes + lane * p.page * 128, map, &bar_full[slot],
                          dh * 64, kvh, 0, cur);
      }
      ++issued;
      if (i & 1) {
        cur = block_of(nxt);  // read a tile ago
        nxt = tile_pages((i >> 1) + 2);
      }
    }
    if (lane == 0 && (stop || *aborted)) {  // let issued copies land before shared memory goes
      *aborted = 1;
      for (int i = issued - kRingSlots < 0 ? 0 : issued - kRingSlots; i < issued; ++i)
        tc::mbar_wait(&bar_full[i % kRingSlots], (i / kRingSlots) & 1, kWaitLimit);
      tc::mbar_wait(&bar_q, 0, kWaitLimit);
    }
  };
  auto mma_role = [&]() {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = tc::idesc_f16(Fmt<T>::value, kTileM, kTileN, 0);
      constexpr uint32_t idesc_pv = tc::idesc_f16(Fmt<T>::value, kTileM, kHeadDim, 1);
      // Descriptor words computed once; a k-step, a query tile or a ring slot
      // moves the start address only, a 32-bit add on the low word. Building
      // descriptors per MMA made this single thread, not the tensor core, the
      // limit on the MMA rate.
      constexpr uint32_t kTileStep = kTileBytes >> 4;
      const uint64_t q_desc = tc::smem_desc_sw128(tc::smem_u32(smem), 16, 1024);  // Q_A, Q_B, P_A, P_B
      const uint64_t k_desc = tc::smem_desc_sw128(tc::smem_u32(ring), 16, 1024);
      const uint64_t v_desc = tc::smem_desc_sw128(tc::smem_u32(ring), kHalfBytes, 1024);
      const uint32_t q_lo = static_cast<uint32_t>(q_desc), q_hi = static_cast<uint32_t>(q_desc >> 32);
      const uint32_t k_lo = static_cast<uint32_t>(k_desc), k_hi = static_cast<uint32_t>(k_desc >> 32);
      const uint32_t v_lo = static_cast<uint32_t>(v_desc), v_hi = static_cast<uint32_t>(v_desc >> 32);
      int commits_s[2] = {0, 0}, commits_pv[2] = {0, 0};
      auto wait_item = [&](int i) {
        return tc::mbar_wait(&bar_full[i % kRingSlots], (i / kRingSlots) & 1, kWaitLimit);
      };
      // k-steps [k0, k1) of S_x = Q_x K^T, K in ring slot `slot`
      auto s_steps = [&](int x, int slot, int k0, int k1) {
        const uint32_t qb = q_lo + x * kTileStep;
        const uint32_t kb = k_lo + slot * kTileStep;
#pragma unroll
        for (int ks = k0; ks < k1; ++ks) {
          const uint32_t off = ((ks >> 2) * kHalfBytes + (ks & 3) * 32) >> 4;
          tc::mma_f16_ss(tmem + x * kTileN, tc::desc64(qb + off, q_hi), tc::desc64(kb + off, k_hi),
                         idesc_qk, ks > 0 ? 1u : 0u);
        }
      };
      // k-steps [k0, k1) of O_x += P_x V, V in ring slot `slot`
      [[maybe_unused]] bool split_tile[2] = {false, false};
      if constexpr (kSplitP) {
        for (int x = 0; x < 2; ++x)
          split_tile[x] = ctx - qlen + m0 + x * kTileM + 1 < p.split_keys;
      }
      auto pv_steps = [&](int x, int slot, int k0, int k1, uint32_t accumulate) {
        const uint32_t vb = v_lo + slot * kTileStep;
#pragma unroll
        for (int ks = k0; ks < k1; ++ks) {
          const uint64_t bdesc = tc::desc64(vb + ks * (2048 >> 4), v_hi);
          const uint32_t acc = ks > 0 ? 1u : accumulate;
          if constexpr (kPTmem) {
            // P_x over S_x's columns, 8 columns (16 keys) per step: the first
            // 64 columns, or with the split softmax each half's P at the start
            // of its own 64 S columns ([0, 32) and [64, 96))
            const uint32_t pcol = ks * 8 + (kHalves == 2 && ks >= 4 ? 32 : 0);
            tc::mma_f16_ts(tmem + 2 * kTileN + x * kHeadDim, tmem + x * kTileN + pcol, bdesc,
                           idesc_pv, acc);
          } else {
            const uint32_t off = ((ks >> 2) * kHalfBytes + (ks & 3) * 32) >> 4;
            tc::mma_f16_ss(tmem + 2 * kTileN + x * kHeadDim,
                           tc::desc64(q_lo + (2 + x) * kTileStep + off, q_hi), bdesc, idesc_pv, acc);
          }
        }
        if constexpr (kSplitP) {
          // the same keys' P_lo, 64 columns further on: one branch per tile
          if (split_tile[x]) {
#pragma unroll
            for (int ks = k0; ks < k1; ++ks)
              tc::mma_f16_ts(tmem + 2 * kTileN + x * kHeadDim, tmem + x * kTileN + 64 + ks * 8,
                             tc::desc64(vb + ks * (2048 >> 4), v_hi), idesc_pv, 1u);
          }
        }
      };
      auto commit_s = [&](int x) {
        tc::mma_commit(&bar_s[x]);
        ++commits_s[x];
      };
      auto commit_pv = [&](int x) {
        tc::mma_commit(&bar_pv[x]);
        ++commits_pv[x];
      };
      // Once P_x(t) is ready: PV_x(t) and, unless t is the last key tile,
      // S_x(t+1). With P in TMEM, P_x(t) occupies S_x's columns, so S_x(t+1)
      // must follow PV_x(t). With P in shared memory, S_x(t+1) goes first
      // (the next softmax of tile x waits on it, not on PV) and the two are
      // interleaved four k-steps at a time: a run of eight MMAs of one
      // B-operand major-ness followed by eight of the other costs the tensor
      // core about 30 cycles per MMA, runs of four or less cost nothing.
      // With P in TMEM, bar_pv is committed after the last PV only: S_x(t+1)
      // follows PV_x(t), and a commit tracks every earlier MMA of this
      // thread, so S_x(t+1) ready already means PV_x(t) is done.
      auto after_p = [&](int x, int v_slot, int k_slot, bool more, uint32_t accumulate) {
        if constexpr (kPTmem) {
          pv_steps(x, v_slot, 0, 8, accumulate);
          if (!more) commit_pv(x);
          if (more) {
            s_steps(x, k_slot, 0, 8);
            commit_s(x);
          }
        } else if (more) {
          s_steps(x, k_slot, 0, 4);
          pv_steps(x, v_slot, 0, 4, accumulate);
          s_steps(x, k_slot, 4, 8);
          commit_s(x);
          pv_steps(x, v_slot, 4, 8, 1u);
          commit_pv(x);
        } else {
          pv_steps(x, v_slot, 0, 8, accumulate);
          commit_pv(x);
        }
      };
      bool ok = tc::mbar_wait(&bar_q, 0, kWaitLimit) && wait_item(0);
      if (ok) {
        tc::tc_fence_after();
        s_steps(0, 0, 0, 8);
        commit_s(0);
        s_steps(1, 0, 0, 8);
        commit_s(1);
        tc::mma_commit(&bar_empty[0]);  // K(0) read by both S MMAs
      }
      // ring slots of V(t) and K(t+1): items 2t+1 and 2t+2
      int v_slot = 1 % kRingSlots;
      for (int t = 0; ok && t < n_tiles; ++t) {
        const int k_next = v_slot + 1 == kRingSlots ? 0 : v_slot + 1;
        const bool more = t + 1 < n_tiles;
        const uint32_t accumulate = t > 0 ? 1u : 0u;
        // the ring items first: they landed long ago, and testing them while
        // the softmax of tile A still runs keeps them off the path from P_A
        // to the MMAs. The P barriers are polled (test_wait, never
        // suspended): this one thread's wake-up is on the critical path.
        ok = wait_item(2 * t + 1) && (!more || wait_item(2 * t + 2));
        if (ok && !more) {
          zero_tail_rows(ring + v_slot * kTileBytes, ctx, t * kTileN, p.page);
          tc::fence_proxy_async_smem();
        }
        ok = ok && tc::mbar_poll(&bar_p[0], t & 1, kWaitLimit);
        if (!ok) break;
        tc::tc_fence_after();
        after_p(0, v_slot, k_next, more, accumulate);
        ok = tc::mbar_poll(&bar_p[1], t & 1, kWaitLimit);
        if (!ok) break;
        tc::tc_fence_after();
        after_p(1, v_slot, k_next, more, accumulate);
        tc::mma_commit(&bar_empty[v_slot]);  // V(t) read by both PV MMAs
        if (more) tc::mma_commit(&bar_empty[k_next]);  // K(t+1) read by both S MMAs
        v_slot = k_next + 1 == kRingSlots ? 0 : k_next + 1;
      }
      if (!ok) {
        *aborted = 1;
        // every commit arrives once all earlier MMAs are done: wait the last
        for (int x = 0; x < 2; ++x) {
          if (commits_pv[x]) tc::mbar_wait(&bar_pv[x], (commits_pv[x] - 1) & 1, kWaitLimit);
          if (commits_s[x]) tc::mbar_wait(&bar_s[x], (commits_s[x] - 1) & 1, kWaitLimit);
        }
      }
    }
  };
  auto softmax_role = [&]() {
    // ---------------- softmax of tile x, one query row per thread; with
    // kHalves = 2 two warps share the rows, one per half of the key columns
    const int x = warp / (4 * kHalves);
    const int h = kHalves == 2 ? (warp >> 2) & 1 : 0;
    const int quarter = warp & 3;  // TMEM lanes [32 quarter, 32 quarter + 32)
    const int r = quarter * 32 + lane;
    const uint32_t pair_id = 1 + x * 4 + quarter;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_tmem = tmem + x * kTileN + h * kCols + lane_base;
    const uint32_t o_tmem = tmem + 2 * kTileN + x * kHeadDim + h * kOCols + lane_base;
    const int qi = m0 + x * kTileM + r;
    const int row_limit = min(ctx - qlen + qi, ctx - 1);
    // warp-uniform: the same rule as the MMA thread's
    [[maybe_unused]] const bool split_tile =
        kSplitP && ctx - qlen + m0 + x * kTileM + 1 < p.split_keys;
    float m_used = -INFINITY;
    float l_sum = 0.f;
    int t = 0;
    for (; t < n_tiles; ++t) {
      // loop exits are warp-uniform (pair-uniform with kHalves = 2): the
      // next statement is a warp-collective tcgen05.ld
      const bool ready = __all_sync(
          kFullMask, *aborted == 0 && tc::mbar_wait(&bar_s[x], t & 1, kWaitLimit));
      if (kHalves == 1 && !ready) {
        *aborted = 1;
        break;
      }
      tc::tc_fence_after();
      const int n0 = t * kTileN + h * kCols;  // this warp's first key
      // keys past the causal limit somewhere in the warp (warp-uniform, so the
      // TMEM collectives below never sit under a divergent branch)
      const bool diagonal = __any_sync(kFullMask, n0 + kCols - 1 > row_limit);
      if constexpr (kWide) {
        // One pass: the row's 128 scores stay in registers from the TMEM
        // load to the P store. Masked scores become -inf, whose exponential
        // is 0, so the probabilities need no mask of their own.
        uint32_t sr[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tc::tmem_ld32(s_tmem + c * 32, sr[c]);
#pragma unroll
        for (int c = 0; c < 4; ++c) tc::tmem_ld_wait(sr[c]);
        if (diagonal) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (n0 + c * 32 + j > row_limit) sr[c][j] = __float_as_uint(-INFINITY);
        }
        float mc[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          mc[c] = -INFINITY;
#pragma unroll
          for (int j = 0; j < 32; j += 2)
            mc[c] = max3(mc[c], __uint_as_float(sr[c][j]), __uint_as_float(sr[c][j + 1]));
        }
        const float mx = fmaxf(fmaxf(mc[0], mc[1]), fmaxf(mc[2], mc[3]));
        const float m_new = fmaxf(m_used, mx * p.scale_log2);
        float factor = 1.f;
        if (m_new > m_used + 8.f) {
          factor = ex2(m_used - m_new);
          m_used = m_new;
        }
        const float neg_mref = m_used == -INFINITY ? 0.f : -m_used;
        // PV_x(t-1) is done (S_x(t) was issued after it): rescale O_x
        if (t > 0 && __any_sync(kFullMask, factor != 1.f)) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tc::tmem_ld32(o_tmem + c * 32, o);
            tc::tmem_ld_wait(o);
#pragma unroll
            for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * factor);
            tc::tmem_st32(o_tmem + c * 32, o);
          }
          tc::tmem_st_wait();
        }
        const uint64_t scale2 = pk2(p.scale_log2, p.scale_log2);
        const uint64_t neg2 = pk2(neg_mref, neg_mref);
        // P of the row's 128 keys into TMEM; with `split`, P_lo beside it.
        // Two instantiations chosen by one warp-uniform branch, so the common
        // (unsplit) path carries none of the split's registers.
        auto emit_p = [&](auto split) {
          constexpr bool kSplit = decltype(split)::value;
          uint64_t psum2 = pk2(0.f, 0.f);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t packed[16];
            [[maybe_unused]] uint32_t rest[16];  // P_lo
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              const uint64_t arg = fma2(pk2(__uint_as_float(sr[c][j]), __uint_as_float(sr[c][j + 1])),
                                        scale2, neg2);
              float p0, p1;
              upk2(arg, p0, p1);
              if ((j / 2) % 8 < kPolyPairs) {  // this pair on the FMA pipe
                upk2(exp2_poly2(p0, p1), p0, p1);
              } else {
                p0 = ex2(p0);
                p1 = ex2(p1);
              }
              psum2 = add2(psum2, pk2(p0, p1));
              packed[j / 2] = pack2<T>(p0, p1);
              if constexpr (kSplit) {
                float h0, h1;
                unpack2<T>(packed[j / 2], h0, h1);
                rest[j / 2] = pack2<T>(p0 - h0, p1 - h1);
              }
            }
            tc::tmem_st16(s_tmem + c * 16, packed);  // S columns already in registers
            if constexpr (kSplit) tc::tmem_st16(s_tmem + 64 + c * 16, rest);
          }
          return psum2;
        };
        uint64_t psum2;
        if (kSplitP && split_tile)
          psum2 = emit_p(std::integral_constant<bool, kSplitP>{});
        else
          psum2 = emit_p(std::false_type{});
        float lo, hi;
        upk2(psum2, lo, hi);
        l_sum = l_sum * factor + (lo + hi);
      } else {
        // Row max, 64 columns per TMEM wait. The pass exists in two
        // instantiations, with and without the causal mask, chosen by one
        // warp-uniform branch: a mask test inside the unrolled loops was
        // predicated into every key tile, not just the diagonal ones.
        auto row_max = [&](auto masked) {
          constexpr bool kMasked = decltype(masked)::value;
          float m = -INFINITY;
  #pragma unroll
          for (int hb = 0; hb < kCols / 64; ++hb) {
            uint32_t sr[2][32];
            tc::tmem_ld32(s_tmem + hb * 64, sr[0]);
            tc::tmem_ld32(s_tmem + hb * 64 + 32, sr[1]);
            tc::tmem_ld_wait(sr[0]);
            tc::tmem_ld_wait(sr[1]);
            if constexpr (kMasked) {
  #pragma unroll
              for (int c = 0; c < 2; ++c)
  #pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (n0 + hb * 64 + c * 32 + j > row_limit) sr[c][j] = __float_as_uint(-INFINITY);
            }
  #pragma unroll
            for (int c = 0; c < 2; ++c)
  #pragma unroll
              for (int j = 0; j < 32; j += 2)
                m = max3(m, __uint_as_float(sr[c][j]), __uint_as_float(sr[c][j + 1]));
          }
          return m;
        };
        float mx = -INFINITY;
        if (ready) {
          if (diagonal)
            mx = row_max(std::true_type{});
          else
            mx = row_max(std::false_type{});
        }
        if constexpr (kHalves == 2) {
          // both halves take the larger maximum (fmaxf is exact and symmetric,
          // so the two warps hold the same base, factor and P scale)
          pair_red[(x * 2 + h) * kTileM + r] = mx;
          if (!pair_barrier_and(pair_id, ready)) {
            *aborted = 1;
            break;
          }
          mx = fmaxf(mx, pair_red[(x * 2 + (h ^ 1)) * kTileM + r]);
        }
        const float m_new = fmaxf(m_used, mx * p.scale_log2);
        float factor = 1.f;
        if (m_new > m_used + 8.f) {
          factor = ex2(m_used - m_new);
          m_used = m_new;
        }
        const float neg_mref = m_used == -INFINITY ? 0.f : -m_used;
        // PV(t-1) must be done: it read P_x and it wrote O_x. With P in TMEM
        // the S_x(t) completion seen above implies it (S_x(t) was issued after
        // PV_x(t-1)). A timed-out wait marks the call aborted and skips the
        // rescale; the next key tile's readiness test then ends the loop (for
        // both warps of a pair).
        if (t > 0) {
          if (!kPTmem &&
              !__all_sync(kFullMask, tc::mbar_wait(&bar_pv[x], (t - 1) & 1, kWaitLimit))) {
            *aborted = 1;
          } else {
            tc::tc_fence_after();
            if (__any_sync(kFullMask, factor != 1.f)) {  // warp-collective TMEM access
  #pragma unroll
              for (int c = 0; c < kOCols / 32; ++c) {
                uint32_t o[32];
                tc::tmem_ld32(o_tmem + c * 32, o);
                tc::tmem_ld_wait(o);
  #pragma unroll
                for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * factor);
                tc::tmem_st32(o_tmem + c * 32, o);
              }
              tc::tmem_st_wait();
            }
          }
        }
        // probabilities p = 2^(s * scale_log2 - m) -> P_x, row sum. Every
        // exponential runs on the MUFU unit: a polynomial on the FMA pipe needs
        // integer and min/max work on the ALU pipe, which the row max and the
        // P conversion already keep busy, and measured slower at every split
        // tried (1/8 to 1/2 of the columns). Arguments and sums use packed
        // fp32x2 ops.
        const uint64_t scale2 = pk2(p.scale_log2, p.scale_log2);
        const uint64_t neg2 = pk2(neg_mref, neg_mref);
        auto probabilities = [&](auto masked) {
          constexpr bool kMasked = decltype(masked)::value;
          uint64_t psum2 = pk2(0.f, 0.f);
  #pragma unroll
          for (int cc = 0; cc < kCols / 32; ++cc) {  // 32-column chunks
            uint32_t sr[32];
            tc::tmem_ld32(s_tmem + cc * 32, sr);
            tc::tmem_ld_wait(sr);
            uint32_t packed[16];
  #pragma unroll
            for (int j = 0; j < 32; j += 2) {
              const uint64_t arg =
                  fma2(pk2(__uint_as_float(sr[j]), __uint_as_float(sr[j + 1])), scale2, neg2);
              float p0, p1;
              upk2(arg, p0, p1);
              p0 = ex2(p0);
              p1 = ex2(p1);
              if constexpr (kMasked) {
                const int key = n0 + cc * 32 + j;
                p0 = key <= row_limit ? p0 : 0.f;
                p1 = key + 1 <= row_limit ? p1 : 0.f;
              }
              psum2 = add2(psum2, pk2(p0, p1));
              packed[j / 2] = pack2<T>(p0, p1);
            }
            if constexpr (kPTmem) {
              // P columns [16 cc, 16 cc + 16) of this warp's S columns: ones
              // this thread already read
              tc::tmem_st16(s_tmem + cc * 16, packed);
            } else {
              uint8_t* base = smem + (2 + x) * kTileBytes + (cc >> 1) * kHalfBytes;  // P_x
  #pragma unroll
              for (int v = 0; v < 4; ++v)
                *reinterpret_cast<uint4*>(base + sw128(r, (cc & 1) * 4 + v)) =
                    make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
            }
          }
          float lo, hi;
          upk2(psum2, lo, hi);
          return lo + hi;
        };
        float psum;
        if (diagonal)
          psum = probabilities(std::true_type{});
        else
          psum = probabilities(std::false_type{});
        l_sum = l_sum * factor + psum;
      }
      if constexpr (kPTmem)
        tc::tmem_st_wait();
      else
        tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      __syncwarp();  // every lane's P is written before the warp's single arrival
      if (lane == 0) tc::mbar_arrive(&bar_p[x]);
    }
    if (t == n_tiles) {
      // the last PV_x: the only commit of bar_pv with P in TMEM
      const uint32_t pv_phase = kPTmem ? 0u : static_cast<uint32_t>((n_tiles - 1) & 1);
      if (!__all_sync(kFullMask, tc::mbar_wait(&bar_pv[x], pv_phase, kWaitLimit)))
        *aborted = 1;
      tc::tc_fence_after();
      if constexpr (kHalves == 2) {
        // row sum of both halves. The partner read this slot's max before its
        // last P arrival, which precedes the PV commit waited on above.
        pair_red[(x * 2 + h) * kTileM + r] = l_sum;
        pair_barrier(pair_id);
        l_sum = pair_red[x * 2 * kTileM + r] + pair_red[(x * 2 + 1) * kTileM + r];
      }
    }
    // epilogue (l_sum is in a register): warp-collective TMEM reads of O_x
    if (t == n_tiles && !__any_sync(kFullMask, *aborted != 0)) {
      const bool store = qi < qlen;
      T* dst = static_cast<T*>(p.out) + (qbegin + (store ? qi : 0)) * p.o_rs + head * p.o_hs +
               h * kOCols;
      const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
#pragma unroll
      for (int c = 0; c < kOCols / 32; ++c) {
        uint32_t o[32];
        tc::tmem_ld32(o_tmem + c * 32, o);
        tc::tmem_ld_wait(o);
        if (!store) continue;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint4 w;
          w.x = pack2<T>(__uint_as_float(o[v * 8 + 0]) * inv, __uint_as_float(o[v * 8 + 1]) * inv);
          w.y = pack2<T>(__uint_as_float(o[v * 8 + 2]) * inv, __uint_as_float(o[v * 8 + 3]) * inv);
          w.z = pack2<T>(__uint_as_float(o[v * 8 + 4]) * inv, __uint_as_float(o[v * 8 + 5]) * inv);
          w.w = pack2<T>(__uint_as_float(o[v * 8 + 6]) * inv, __uint_as_float(o[v * 8 + 7]) * inv);
          *reinterpret_cast<uint4*>(dst + c * 32 + v * 8) = w;
        }
      }
    }
  };
  auto zero_rows = [&]() {
    // rows that see no keys: zeros
    const int qi = m0 + (warp >> 2) * kTileM + (tid & (kTileM - 1));
    if (qi < qlen) {
      T* dst = static_cast<T*>(p.out) + (qbegin + qi) * p.o_rs + head * p.o_hs;
      for (int c = 0; c < kHeadDim; c += 8) *reinterpret_cast<uint4*>(dst + c) = make_uint4(0, 0, 0, 0);
    }
  };
  if constexpr (kWide) {
    // Register reallocation per warpgroup, each from one instruction inside
    // its warpgroup's branch so that the role code below it is compiled to
    // the new limit: warpgroups 0-1 (softmax) rise, warpgroup 2 (MMA,
    // producer, two idle warps) drops.
    if (warp >= 8) {
      tc::setmaxnreg_dec<kWideOtherRegs>();
      if (active && warp == kProducerWarp)
        producer_role();
      else if (active && warp == kMmaWarp)
        mma_role();
    } else {
      tc::setmaxnreg_inc<kWideSoftRegs>();
      if (active)
        softmax_role();
      else if (seq >= 0 && n_tiles == 0)
        zero_rows();
    }
  } else {
    if (active && warp == kProducerWarp)
      producer_role();
    else if (active && warp == kMmaWarp)
      mma_role();
    else if (active && warp < kSoftWarps)
      softmax_role();
    else if (seq >= 0 && n_tiles == 0 && warp < 8)
      zero_rows();
  }
  __syncthreads();
  if (*aborted && tid == 0) raise_status(p.status, kStatusTimeout);
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kPairTmemCols);
  }
}

// Whether this CTA's query tile A sees fewer than p.split_keys keys (its
// rows then split P). Every warp finds the CTA's tile by itself, as
// find_tile does (warp shuffles only), so the choice needs no shared memory
// and no barrier.
__device__ __forceinline__ bool cta_needs_split(const PrefillTcParams& p) {
  const int lane = threadIdx.x & 31;
  int running = 0, seq = -1, m0 = 0;
  for (int base = 0; base < p.num_seqs && seq < 0; base += 32) {  // as find_tile
    const int sq = base + lane;
    int tiles = 0;
    if (sq < p.num_seqs) {
      const int qlen = p.cu[sq + 1] - p.cu[sq];
      tiles = qlen > 0 ? (qlen + kPairRows - 1) / kPairRows : 0;
    }
    int incl = tiles;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(kFullMask, incl, o);
      if (lane >= o) incl += y;
    }
    const int excl = running + incl - tiles;
    const int target = static_cast<int>(blockIdx.x);
    const bool mine = sq < p.num_seqs && target >= excl && target < excl + tiles;
    const unsigned hit = __ballot_sync(kFullMask, mine);
    if (hit) {
      const int src = __ffs(hit) - 1;
      seq = __shfl_sync(kFullMask, sq, src);
      const int idx = __shfl_sync(kFullMask, tiles - 1 - (target - excl), src);  // heavy first
      m0 = idx * kPairRows;
    }
    running += __shfl_sync(kFullMask, incl, 31);
  }
  if (seq < 0) return false;
  const int qlen = p.cu[seq + 1] - p.cu[seq];
  return p.lengths[seq] - qlen + m0 + 1 < p.split_keys;
}

// The kernel: CTAs whose query tile A sees fewer than p.split_keys keys (tile
// B sees more) run the body that can split P; all others run the body
// compiled without it, so the common path carries none of the split's
// registers or branches.
template <typename T, bool kPTmem, int kHalves, bool kWide, bool kSplitP = false>
__global__ void __launch_bounds__(pair_threads(kHalves, kWide), 1)
    paged_prefill_tc2_kernel(const __grid_constant__ PrefillTcParams p) {
  if constexpr (kSplitP) {
    if (cta_needs_split(p)) {
      pair_body<T, kPTmem, kHalves, kWide, true>(p);
      return;
    }
  }
  pair_body<T, kPTmem, kHalves, kWide, false>(p);
}

// ---- version 8: 64-key steps, two S buffers per query tile ----------------
//
// The two-tile kernel above chains, per query tile and 128-key step: S ready
// -> softmax -> P -> PV and the next S (16 MMAs) -> S ready, because P lives
// in S's TMEM columns and TMEM (2 x S + 2 x O = 512 columns) has no room for
// a second S. With 64-key steps an S tile is 64 columns, so each query tile
// keeps two S buffers in the same 512 columns (S_A0, S_A1, S_B0, S_B1 in
// [0, 256), O_A and O_B in [256, 512)): the MMA thread issues S_x(t+2) into
// buffer t % 2 right after PV_x(t) has read P_x(t) from it, so S_x(t+1) is
// already computed while the softmax of step t runs and the MMA latency and
// the two hand-offs leave the per-step chain. P_x(t) (and with the split its
// P_lo) overwrite the first 32 (64) columns of their S buffer. A rescale of
// O_x (the lazy base moved) waits for PV_x(t-1) on bar_pv, which the MMA
// thread now commits after every PV (S_x(t) no longer follows PV_x(t-1)).
// K and V of a step are 16 KiB items in a 10-slot ring, consumed in the MMA
// order K(0), K(1), then V(t), K(t+2) for t = 0, 1, ...
//
// Measured on the configs[3] workload: 749-788 TFLOP/s against 898-920 for
// version 6 (~2,900 cycles per 64-key step against ~1,850 per 64 keys). With
// N = 64 the S product re-reads the Q tile from shared memory twice as often
// per key: a step moves ~128 KB of MMA operands plus 32 KB of TMA writes
// through shared memory for 1,024 cycles of tensor work, more than its
// 128 B/clock, so the hand-offs this version removes were not the whole
// limit. It stays selectable (rlt_prefill_tc_select(8)) and parity-tested.
constexpr int kKeys8 = 64;                              // keys per step
constexpr int kItemBytes8 = kKeys8 * kHeadDim * 2;      // K or V of one step: 16 KiB
constexpr int kItemHalf8 = kKeys8 * 128;                // 64 keys x 64 dims: 8 KiB
constexpr int kRingSlots8 = 10;
struct Pair8Shared {
  uint64_t bar_q, bar_full[kRingSlots8], bar_empty[kRingSlots8];
  // per (query tile x, S buffer b) at 2 x + b: S ready, and P written. P
  // has one barrier per buffer because a tile's softmax may finish P_x(t+1)
  // before the MMA thread has polled P_x(t): one barrier would then complete
  // two phases before the poll and its parity would read as not done.
  uint64_t bar_s[4], bar_p[4];
  uint64_t bar_pv[2];
  uint32_t tmem_base;
  int tile_seq, tile_m0, abort_flag;
};
constexpr int kPair8Region = 2 * kTileBytes + kRingSlots8 * kItemBytes8;  // Q_A, Q_B, ring
constexpr int kPair8Slack = kMaxSmem - kPair8Region - static_cast<int>(sizeof(Pair8Shared));
static_assert(kPair8Slack >= 0, "shared memory per CTA (version 8)");

__device__ __forceinline__ bool page_fits_step8(int page) { return page > 0 && kKeys8 % page == 0 && page % 8 == 0; }

template <typename T, bool kSplitP>
__device__ __forceinline__ void pair8_body(const PrefillTcParams& p) {
  constexpr int kMmaWarp = 8;
  constexpr int kProducerWarp = 9;
  extern __shared__ uint8_t smem_raw[];
  const uintptr_t raw = reinterpret_cast<uintptr_t>(smem_raw);
  const uintptr_t skip = ((raw + 1023) & ~static_cast<uintptr_t>(1023)) - raw;
  if (skip > static_cast<uintptr_t>(kPair8Slack) || !page_fits_step8(p.page)) {  // uniform
    if (threadIdx.x == 0) raise_status(p.status, kStatusLayout);
    return;
  }
  uint8_t* smem = smem_raw + skip;
  uint8_t* ring = smem + 2 * kTileBytes;
  Pair8Shared& sh = *reinterpret_cast<Pair8Shared*>(smem + kPair8Region);
  uint64_t& bar_q = sh.bar_q;
  uint64_t* bar_full = sh.bar_full;
  uint64_t* bar_empty = sh.bar_empty;
  uint64_t* bar_s = sh.bar_s;
  uint64_t* bar_p = sh.bar_p;
  uint64_t* bar_pv = sh.bar_pv;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int head = blockIdx.y;
  const int kvh = head / p.group;

  if (warp == 0)
    find_tile<kPairRows, true>(p.cu, p.num_seqs, blockIdx.x, lane, &sh.tile_seq, &sh.tile_m0);
  if (tid == 0) {
    tc::mbar_init(&bar_q, 1);
    for (int i = 0; i < kRingSlots8; ++i) {
      tc::mbar_init(&bar_full[i], 1);
      tc::mbar_init(&bar_empty[i], 1);
    }
    for (int i = 0; i < 4; ++i) {
      tc::mbar_init(&bar_s[i], 1);
      tc::mbar_init(&bar_p[i], 4);  // one arrival per softmax warp of the tile
    }
    for (int x = 0; x < 2; ++x) tc::mbar_init(&bar_pv[x], 1);
    tc::fence_mbar_init();
    sh.abort_flag = 0;
  }
  __syncwarp();
  if (warp == 0) tc::tmem_alloc(&sh.tmem_base, kPairTmemCols);  // warp-collective
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  volatile int* aborted = &sh.abort_flag;

  int seq = sh.tile_seq;
  const int m0 = sh.tile_m0;
  int qbegin = 0, qlen = 0, ctx = 0, n_steps = 0;
  if (seq >= 0) {
    qbegin = p.cu[seq];
    qlen = p.cu[seq + 1] - qbegin;
    ctx = p.lengths[seq];
    if (qbegin < 0 || qlen <= 0 || qbegin + qlen > p.num_tokens || ctx < 0 ||
        static_cast<int64_t>(ctx) > static_cast<int64_t>(p.width) * p.page) {
      if (tid == 0) raise_status(p.status, kStatusBadSequence);
      seq = -1;
    } else {
      const int kmax = ctx - qlen + min(qlen - 1, m0 + kPairRows - 1);
      n_steps = kmax >= 0 ? kmax / kKeys8 + 1 : 0;
    }
  }
  const bool active = seq >= 0 && n_steps > 0;
  // the MMA thread and the softmax warps decide a tile's split alike
  [[maybe_unused]] bool split_tile[2] = {false, false};
  if constexpr (kSplitP) {
    for (int x = 0; x < 2; ++x) split_tile[x] = ctx - qlen + m0 + x * kTileM + 1 < p.split_keys;
  }

  auto producer_role = [&]() {
    // Lane j < pages per step loads page j of an item. Block ids are read a
    // step before their K copy and kept for the V copy two steps later.
    const int ppt = kKeys8 / p.page;
    auto raw_id = [&](int u) {  // INT32_MIN: not a page of the context
      int id = INT32_MIN;
      if (lane < ppt && u < n_steps && (u * ppt + lane) * p.page < ctx)
        id = p.tables[seq * p.t_rs + u * ppt + lane];
      return id;
    };
    auto block_of = [&](int id) {
      int blk = static_cast<int>(p.num_blocks);  // out of range: zero fill
      if (id != INT32_MIN) {
        if (id >= 0 && id < p.num_blocks)
          blk = id;
        else
          raise_status(p.status, kStatusBadBlock);
      }
      return blk;
    };
    if (lane == 0) {
      tc::prefetch_tensormap(&p.qmap);
      tc::prefetch_tensormap(&p.kmap);
      tc::prefetch_tensormap(&p.vmap);
      tc::mbar_expect_tx(&bar_q, 2 * kTileBytes);
      for (int x = 0; x < 2; ++x)
        for (int dh = 0; dh < 2; ++dh)
          tc::tma_load_3d(smem + x * kTileBytes + dh * kHalfBytes, &p.qmap, &bar_q, dh * 64, head,
                          qbegin + m0 + x * kTileM);
    }
    int issued = 0;
    bool stop = false;
    auto emit = [&](bool is_v, int blk) {  // the next ring item
      const int slot = issued % kRingSlots8;
      int ok = 1;
      if (lane == 0)
        ok = *aborted == 0 &&
             (issued < kRingSlots8 ||
              tc::mbar_wait(&bar_empty[slot], (issued / kRingSlots8 - 1) & 1, kWaitLimit));
      if (!__shfl_sync(kFullMask, ok, 0)) {
        stop = true;
        return;
      }
      uint8_t* dst = ring + slot * kItemBytes8;
      const CUtensorMap* map = is_v ? &p.vmap : &p.kmap;
      if (lane == 0) tc::mbar_expect_tx(&bar_full[slot], kItemBytes8);
      __syncwarp();
      if (lane < ppt) {
#pragma unroll
        for (int dh = 0; dh < 2; ++dh)
          tc::tma_load_4d(dst + dh * kItemHalf8 + lane * p.page * 128, map, &bar_full[slot],
                          dh * 64, kvh, 0, blk);
      }
      ++issued;
    };
    int f0 = block_of(raw_id(0));  // blocks of the steps whose K is out and V is not
    int f1 = 0;
    int pending = raw_id(1);
    emit(false, f0);
    if (!stop && n_steps > 1) {
      f1 = block_of(pending);
      pending = raw_id(2);
      emit(false, f1);
    }
    for (int t = 0; !stop && t < n_steps; ++t) {
      emit(true, f0);
      f0 = f1;
      if (!stop && t + 2 < n_steps) {
        f1 = block_of(pending);
        pending = raw_id(t + 3);
        emit(false, f1);
      }
    }
    if (lane == 0 && (stop || *aborted)) {  // let issued copies land before shared memory goes
      *aborted = 1;
      for (int i = issued - kRingSlots8 < 0 ? 0 : issued - kRingSlots8; i < issued; ++i)
        tc::mbar_wait(&bar_full[i % kRingSlots8], (i / kRingSlots8) & 1, kWaitLimit);
      tc::mbar_wait(&bar_q, 0, kWaitLimit);
    }
  };

  auto mma_role = [&]() {
    if (lane != 0) return;
    constexpr uint32_t idesc_qk = tc::idesc_f16(Fmt<T>::value, kTileM, kKeys8, 0);
    constexpr uint32_t idesc_pv = tc::idesc_f16(Fmt<T>::value, kTileM, kHeadDim, 1);
    const uint64_t q_desc = tc::smem_desc_sw128(tc::smem_u32(smem), 16, 1024);
    const uint64_t k_desc = tc::smem_desc_sw128(tc::smem_u32(ring), 16, 1024);
    const uint64_t v_desc = tc::smem_desc_sw128(tc::smem_u32(ring), kItemHalf8, 1024);
    const uint32_t q_lo = static_cast<uint32_t>(q_desc), q_hi = static_cast<uint32_t>(q_desc >> 32);
    const uint32_t k_lo = static_cast<uint32_t>(k_desc), k_hi = static_cast<uint32_t>(k_desc >> 32);
    const uint32_t v_lo = static_cast<uint32_t>(v_desc), v_hi = static_cast<uint32_t>(v_desc >> 32);
    int commits_s[4] = {0, 0, 0, 0}, commits_pv[2] = {0, 0};
    auto wait_item = [&](int i) {
      return tc::mbar_wait(&bar_full[i % kRingSlots8], (i / kRingSlots8) & 1, kWaitLimit);
    };
    // S_x into buffer b = Q_x K^T (M 128, N 64 keys, K 128 dims), K in slot `slot`
    auto s_mma = [&](int x, int b, int slot) {
      const uint32_t qb = q_lo + x * (kTileBytes >> 4);
      const uint32_t kb = k_lo + slot * (kItemBytes8 >> 4);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t q_off = ((ks >> 2) * kHalfBytes + (ks & 3) * 32) >> 4;
        const uint32_t k_off = ((ks >> 2) * kItemHalf8 + (ks & 3) * 32) >> 4;
        tc::mma_f16_ss(tmem + x * 128 + b * kKeys8, tc::desc64(qb + q_off, q_hi),
                       tc::desc64(kb + k_off, k_hi), idesc_qk, ks > 0 ? 1u : 0u);
      }
      tc::mma_commit(&bar_s[2 * x + b]);
      ++commits_s[2 * x + b];
    };
    // O_x += P_x V over the step's 64 keys (P in buffer b's first columns)
    auto pv_mma = [&](int x, int b, int slot, uint32_t accumulate) {
      const uint32_t vb = v_lo + slot * (kItemBytes8 >> 4);
      const uint32_t p_col = tmem + x * 128 + b * kKeys8;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        tc::mma_f16_ts(tmem + 256 + x * kHeadDim, p_col + ks * 8,
                       tc::desc64(vb + ks * (2048 >> 4), v_hi), idesc_pv, ks > 0 ? 1u : accumulate);
      if constexpr (kSplitP) {
        if (split_tile[x]) {
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            tc::mma_f16_ts(tmem + 256 + x * kHeadDim, p_col + 32 + ks * 8,
                           tc::desc64(vb + ks * (2048 >> 4), v_hi), idesc_pv, 1u);
        }
      }
      tc::mma_commit(&bar_pv[x]);
      ++commits_pv[x];
    };
    bool ok = tc::mbar_wait(&bar_q, 0, kWaitLimit) && wait_item(0);
    int item = 0;
    if (ok) {
      tc::tc_fence_after();
      s_mma(0, 0, 0);
      s_mma(1, 0, 0);
      tc::mma_commit(&bar_empty[0]);  // K(0) read by both S MMAs
      item = 1;
      if (n_steps > 1) {
        ok = wait_item(1);
        if (ok) {
          tc::tc_fence_after();
          s_mma(0, 1, 1 % kRingSlots8);
          s_mma(1, 1, 1 % kRingSlots8);
          tc::mma_commit(&bar_empty[1 % kRingSlots8]);
          item = 2;
        }
      }
    }
    for (int t = 0; ok && t < n_steps; ++t) {
      const int b = t & 1;
      const int v_item = item++;
      const int v_slot = v_item % kRingSlots8;
      const bool more = t + 2 < n_steps;
      const int k_item = more ? item++ : -1;
      const int k_slot = more ? k_item % kRingSlots8 : 0;
      ok = wait_item(v_item) && (!more || wait_item(k_item));
      if (ok && t == n_steps - 1) {
        // V rows past the context of its last page may hold any bits (NaN
        // included) and P is 0 there: zero them so P V stays finite
        uint8_t* vt = ring + v_slot * kItemBytes8;
        const int r0 = ctx - t * kKeys8;
        const int page_end = (ctx + p.page - 1) / p.page * p.page;
        const int r1 = min(kKeys8, page_end - t * kKeys8);
        for (int r = max(r0, 0); r < r1; ++r)
#pragma unroll
          for (int half = 0; half < 2; ++half)
#pragma unroll
            for (int c = 0; c < 8; ++c)
              *reinterpret_cast<uint4*>(vt + half * kItemHalf8 + r * 128 + c * 16) =
                  make_uint4(0, 0, 0, 0);
        tc::fence_proxy_async_smem();
      }
      for (int x = 0; ok && x < 2; ++x) {
        ok = tc::mbar_poll(&bar_p[2 * x + b], (t >> 1) & 1, kWaitLimit);
        if (!ok) break;
        tc::tc_fence_after();
        pv_mma(x, b, v_slot, t > 0 ? 1u : 0u);
        if (more) s_mma(x, b, k_slot);  // S_x(t+2) into the buffer PV_x(t) just read
      }
      if (!ok) break;
      tc::mma_commit(&bar_empty[v_slot]);  // V(t) read by both PV MMAs
      if (more) tc::mma_commit(&bar_empty[k_slot]);  // K(t+2) read by both S MMAs
    }
    if (!ok) {
      *aborted = 1;
      // every commit arrives once all earlier MMAs are done: wait for the
      // last two phases of each barrier in order
      auto drain = [&](uint64_t* bar, int commits) {
        if (commits > 1) tc::mbar_wait(bar, (commits - 2) & 1, kWaitLimit);
        if (commits > 0) tc::mbar_wait(bar, (commits - 1) & 1, kWaitLimit);
      };
      for (int x = 0; x < 2; ++x) drain(&bar_pv[x], commits_pv[x]);
      for (int i = 0; i < 4; ++i) drain(&bar_s[i], commits_s[i]);
    }
  };

  auto softmax_role = [&]() {
    const int x = warp >> 2;
    const int quarter = warp & 3;  // TMEM lanes [32 quarter, 32 quarter + 32)
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t o_tmem = tmem + 256 + x * kHeadDim + lane_base;
    const int qi = m0 + x * kTileM + r;
    const int row_limit = min(ctx - qlen + qi, ctx - 1);
    float m_used = -INFINITY;
    float l_sum = 0.f;
    int t = 0;
    for (; t < n_steps; ++t) {
      const int b = t & 1;
      const bool ready = __all_sync(
          kFullMask, *aborted == 0 && tc::mbar_wait(&bar_s[2 * x + b], (t >> 1) & 1, kWaitLimit));
      if (!ready) {
        *aborted = 1;
        break;
      }
      tc::tc_fence_after();
      const uint32_t s_tmem = tmem + x * 128 + b * kKeys8 + lane_base;
      const int n0 = t * kKeys8;
      const bool diagonal = __any_sync(kFullMask, n0 + kKeys8 - 1 > row_limit);
      uint32_t sr[2][32];
      tc::tmem_ld32(s_tmem, sr[0]);
      tc::tmem_ld32(s_tmem + 32, sr[1]);
      tc::tmem_ld_wait(sr[0]);
      tc::tmem_ld_wait(sr[1]);
      if (diagonal) {
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (n0 + c * 32 + j > row_limit) sr[c][j] = __float_as_uint(-INFINITY);
      }
      float mc[2];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        mc[c] = -INFINITY;
#pragma unroll
        for (int j = 0; j < 32; j += 2)
          mc[c] = max3(mc[c], __uint_as_float(sr[c][j]), __uint_as_float(sr[c][j + 1]));
      }
      const float m_new = fmaxf(m_used, fmaxf(mc[0], mc[1]) * p.scale_log2);
      float factor = 1.f;
      if (m_new > m_used + 8.f) {
        factor = ex2(m_used - m_new);
        m_used = m_new;
      }
      const float neg_mref = m_used == -INFINITY ? 0.f : -m_used;
      if (t > 0 && __any_sync(kFullMask, factor != 1.f)) {
        // O_x is quiescent once PV_x(t-1) is done. S_x(t) ready implies
        // PV_x(t-2) done (S_x(t) followed it into the same buffer), so the
        // barrier is in phase t-1 or past it and one parity wait is exact.
        if (!__all_sync(kFullMask, tc::mbar_wait(&bar_pv[x], (t - 1) & 1, kWaitLimit))) {
          *aborted = 1;
          break;
        }
        tc::tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tc::tmem_ld32(o_tmem + c * 32, o);
          tc::tmem_ld_wait(o);
#pragma unroll
          for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * factor);
          tc::tmem_st32(o_tmem + c * 32, o);
        }
        tc::tmem_st_wait();
      }
      const uint64_t scale2 = pk2(p.scale_log2, p.scale_log2);
      const uint64_t neg2 = pk2(neg_mref, neg_mref);
      auto emit_p = [&](auto split) {
        constexpr bool kSplit = decltype(split)::value;
        uint64_t psum2 = pk2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t packed[16];
          [[maybe_unused]] uint32_t rest[16];  // P_lo
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const uint64_t arg =
                fma2(pk2(__uint_as_float(sr[c][j]), __uint_as_float(sr[c][j + 1])), scale2, neg2);
            float p0, p1;
            upk2(arg, p0, p1);
            p0 = ex2(p0);
            p1 = ex2(p1);
            psum2 = add2(psum2, pk2(p0, p1));
            packed[j / 2] = pack2<T>(p0, p1);
            if constexpr (kSplit) {
              float h0, h1;
              unpack2<T>(packed[j / 2], h0, h1);
              rest[j / 2] = pack2<T>(p0 - h0, p1 - h1);
            }
          }
          tc::tmem_st16(s_tmem + c * 16, packed);  // S columns already in registers
          if constexpr (kSplit) tc::tmem_st16(s_tmem + 32 + c * 16, rest);
        }
        return psum2;
      };
      uint64_t psum2;
      if (kSplitP && split_tile[x])
        psum2 = emit_p(std::integral_constant<bool, kSplitP>{});
      else
        psum2 = emit_p(std::false_type{});
      float lo, hi;
      upk2(psum2, lo, hi);
      l_sum = l_sum * factor + (lo + hi);
      tc::tmem_st_wait();
      tc::tc_fence_before();
      __syncwarp();  // every lane's P is written before the warp's single arrival
      if (lane == 0) tc::mbar_arrive(&bar_p[2 * x + b]);
    }
    if (t == n_steps) {
      // S_x(n-1) ready implied PV_x(n-3) done, so PV_x(n-2) and PV_x(n-1) may
      // both be pending: wait for their phases in order (one wait on the last
      // parity alone would match the completed phase n-3)
      bool done = n_steps < 2 || tc::mbar_wait(&bar_pv[x], (n_steps - 2) & 1, kWaitLimit);
      done = done && tc::mbar_wait(&bar_pv[x], (n_steps - 1) & 1, kWaitLimit);
      if (!__all_sync(kFullMask, done)) *aborted = 1;
      tc::tc_fence_after();
    }
    if (t == n_steps && !__any_sync(kFullMask, *aborted != 0)) {
      const bool store = qi < qlen;
      T* dst = static_cast<T*>(p.out) + (qbegin + (store ? qi : 0)) * p.o_rs + head * p.o_hs;
      const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
#pragma unroll
      for (int c = 0; c < kHeadDim / 32; ++c) {
        uint32_t o[32];
        tc::tmem_ld32(o_tmem + c * 32, o);
        tc::tmem_ld_wait(o);
        if (!store) continue;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint4 w;
          w.x = pack2<T>(__uint_as_float(o[v * 8 + 0]) * inv, __uint_as_float(o[v * 8 + 1]) * inv);
          w.y = pack2<T>(__uint_as_float(o[v * 8 + 2]) * inv, __uint_as_float(o[v * 8 + 3]) * inv);
          w.z = pack2<T>(__uint_as_float(o[v * 8 + 4]) * inv, __uint_as_float(o[v * 8 + 5]) * inv);
          w.w = pack2<T>(__uint_as_float(o[v * 8 + 6]) * inv, __uint_as_float(o[v * 8 + 7]) * inv);
          *reinterpret_cast<uint4*>(dst + c * 32 + v * 8) = w;
        }
      }
    }
  };
  auto zero_rows = [&]() {
    const int qi = m0 + (warp >> 2) * kTileM + (tid & (kTileM - 1));
    if (qi < qlen) {
      T* dst = static_cast<T*>(p.out) + (qbegin + qi) * p.o_rs + head * p.o_hs;
      for (int c = 0; c < kHeadDim; c += 8) *reinterpret_cast<uint4*>(dst + c) = make_uint4(0, 0, 0, 0);
    }
  };
  if (warp >= 8) {
    tc::setmaxnreg_dec<kWideOtherRegs>();
    if (active && warp == kProducerWarp)
      producer_role();
    else if (active && warp == kMmaWarp)
      mma_role();
  } else {
    tc::setmaxnreg_inc<kWideSoftRegs>();
    if (active)
      softmax_role();
    else if (seq >= 0 && n_steps == 0)
      zero_rows();
  }
  __syncthreads();
  if (*aborted && tid == 0) raise_status(p.status, kStatusTimeout);
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kPairTmemCols);
  }
}

// Version 8 kernel: the same per-CTA choice between the split and unsplit
// bodies as version 6 (the split only where query tile A sees fewer than
// p.split_keys keys).
template <typename T, bool kSplitP>
__global__ void __launch_bounds__(pair_threads(1, true), 1)
    paged_prefill_tc8_kernel(const __grid_constant__ PrefillTcParams p) {
  if constexpr (kSplitP) {
    if (cta_needs_split(p)) {
      pair8_body<T, true>(p);
      return;
    }
  }
  pair8_body<T, false>(p);
}

// ---- host side --------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

bool encode(CUtensorMap* map, CUtensorMapDataType type, uint32_t rank, const void* base,
            const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const uint32_t elem[4] = {1, 1, 1, 1};
  return fn(map, type, rank, const_cast<void*>(base), dims, strides_bytes, box, elem,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

// Which tensor-core kernel rlt_paged_prefill launches: 6 (default) = 5 with
// bf16 P split into hi + lo in the query tiles that attend few keys, 7 = 5
// with P split everywhere, 5 = warp-specialised two-tile kernel with P in
// TMEM and register-resident scores, 4 = split softmax (two warps per row
// set), 3 = one warp per row set reading S from TMEM twice, 2 = as 3 with P
// in shared memory, 1 = the single-tile kernel, 8 = 6 with 64-key steps and
// two S buffers per query tile (pages of 8 to 64 tokens; 128-token pages run
// 6). 6 costs no measurable time over 5 on the configs[3] workload (CTAs
// without a splitting tile run a body compiled without the split).
std::atomic<int> g_prefill_version{6};
// Version 6 splits P in query tiles whose first row sees fewer keys than
// this; over more keys the bf16 roundings of P average out (error ~ 2^-9 x
// 1.6 / sqrt(keys) per output at unit-variance scores, below 1e-4 here).
constexpr int kSplitKeys = 512;

template <typename T, bool kSplitP>
cudaError_t launch_pair8(dim3 grid, const PrefillTcParams& p, cudaStream_t stream) {
  auto kernel = paged_prefill_tc8_kernel<T, kSplitP>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [kernel] {
    attr_err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
    if (attr_err == cudaSuccess) {
      // the register split assumes this launch allocation (as launch_pair)
      cudaFuncAttributes attr{};
      attr_err = cudaFuncGetAttributes(&attr, kernel);
      if (attr_err == cudaSuccess && attr.numRegs < kWideLaunchRegs)
        attr_err = cudaErrorInvalidConfiguration;
    }
  });
  if (attr_err != cudaSuccess) return attr_err;
  kernel<<<grid, pair_threads(1, true), kMaxSmem, stream>>>(p);
  return cudaSuccess;
}

template <typename T, bool kPTmem, int kHalves, bool kWide = false, bool kSplitP = false>
cudaError_t launch_pair(dim3 grid, const PrefillTcParams& p, cudaStream_t stream) {
  constexpr int bytes = PairLayout<kPTmem>::kSmemBytes;
  auto kernel = paged_prefill_tc2_kernel<T, kPTmem, kHalves, kWide, kSplitP>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [kernel] {
    attr_err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (kWide && attr_err == cudaSuccess) {
      // the register split assumes this launch allocation; with fewer
      // registers the softmax warpgroups' increase could never be granted
      cudaFuncAttributes attr{};
      attr_err = cudaFuncGetAttributes(&attr, kernel);
      if (attr_err == cudaSuccess && attr.numRegs < kWideLaunchRegs)
        attr_err = cudaErrorInvalidConfiguration;
    }
  });
  if (attr_err != cudaSuccess) return attr_err;
  kernel<<<grid, pair_threads(kHalves, kWide), bytes, stream>>>(p);
  return cudaSuccess;
}

}  // namespace

namespace detail {

constexpr int kNotEligible = 1;

// A 4-D tiled tensor map over one layer view of a KV pool, [blocks, page,
// Hkv, D] with element strides (bs, ts, hs), box {64, 1, page, 1}, 128-byte
// swizzle: one TMA load brings 64 head dims of one KV head for every token
// of one page. False when the driver rejects the shape or strides.
bool encode_kv_page_map(CUtensorMap* map, int32_t dtype, const void* base, int32_t head_dim,
                        int32_t hkv, int32_t page, int64_t num_blocks, int64_t bs, int64_t ts,
                        int64_t hs) {
  const CUtensorMapDataType type =
      dtype == RLT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const uint64_t dims[4] = {static_cast<uint64_t>(head_dim), static_cast<uint64_t>(hkv),
                            static_cast<uint64_t>(page), static_cast<uint64_t>(num_blocks)};
  const uint64_t strides[3] = {static_cast<uint64_t>(hs) * 2, static_cast<uint64_t>(ts) * 2,
                               static_cast<uint64_t>(bs) * 2};
  const uint32_t box[4] = {64, 1, static_cast<uint32_t>(page), 1};
  return encode(map, type, 4, base, dims, strides, box);
}

bool prefill_tc_shape(int32_t dtype, int32_t head_dim, int32_t page) {
  return (dtype == RLT_BF16 || dtype == RLT_F16) && head_dim == kHeadDim &&
         (page == 8 || page == 16 || page == 32 || page == 64 || page == 128);
}

// Launch the tensor-core prefill when the shape fits it; kNotEligible leaves
// the call to the CUDA-core path.
int paged_prefill_tc(const void* q, const void* key_cache, const void* value_cache,
                     const int32_t* block_tables, const int32_t* context_lengths,
                     const int32_t* cu_seqlens_q, void* out, int32_t* status, int32_t dtype,
                     int32_t num_tokens, int32_t num_seqs, int32_t hq, int32_t hkv,
                     int32_t head_dim, int32_t page, int32_t width, int64_t num_blocks,
                     const int64_t* st, float scale, cudaStream_t stream) {
  // st: q_rs, q_hs, k_bs, k_ts, k_hs, v_bs, v_ts, v_hs, t_rs, o_rs, o_hs (elements)
  if (!prefill_tc_shape(dtype, head_dim, page)) return kNotEligible;
  if (num_blocks <= 0 || num_blocks >= INT32_MAX || num_seqs <= 0) return kNotEligible;
  if (!aligned16(q) || !aligned16(key_cache) || !aligned16(value_cache) || !aligned16(out))
    return kNotEligible;
  for (int i = 0; i < 11; ++i)
    if (i != 8 && (st[i] * 2) % 16) return kNotEligible;
  if (st[0] <= 0 || st[1] <= 0 || st[2] <= 0 || st[3] <= 0 || st[4] <= 0 || st[5] <= 0 ||
      st[6] <= 0 || st[7] <= 0)
    return kNotEligible;

  PrefillTcParams p{};
  const CUtensorMapDataType type =
      dtype == RLT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(head_dim), static_cast<uint64_t>(hq),
                              static_cast<uint64_t>(num_tokens)};
    const uint64_t strides[2] = {static_cast<uint64_t>(st[1]) * 2, static_cast<uint64_t>(st[0]) * 2};
    const uint32_t box[3] = {64, 1, kTileM};
    if (!encode(&p.qmap, type, 3, q, dims, strides, box)) return kNotEligible;
  }
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(head_dim), static_cast<uint64_t>(hkv),
                              static_cast<uint64_t>(page), static_cast<uint64_t>(num_blocks)};
    const uint32_t box[4] = {64, 1, static_cast<uint32_t>(page), 1};
    const uint64_t ks[3] = {static_cast<uint64_t>(st[4]) * 2, static_cast<uint64_t>(st[3]) * 2,
                            static_cast<uint64_t>(st[2]) * 2};
    const uint64_t vs[3] = {static_cast<uint64_t>(st[7]) * 2, static_cast<uint64_t>(st[6]) * 2,
                            static_cast<uint64_t>(st[5]) * 2};
    if (!encode(&p.kmap, type, 4, key_cache, dims, ks, box)) return kNotEligible;
    if (!encode(&p.vmap, type, 4, value_cache, dims, vs, box)) return kNotEligible;
  }
  p.tables = block_tables;
  p.lengths = context_lengths;
  p.cu = cu_seqlens_q;
  p.out = out;
  p.status = status;
  p.num_seqs = num_seqs;
  p.num_tokens = num_tokens;
  p.hq = hq;
  p.group = hq / hkv;
  p.page = page;
  p.width = width;
  p.num_blocks = num_blocks;
  p.t_rs = st[8];
  p.o_rs = st[9];
  p.o_hs = st[10];
  p.scale_log2 = scale * 1.4426950408889634f;
  const int version = g_prefill_version.load();
  p.split_keys = version == 7 ? INT32_MAX : kSplitKeys;

  if (version == 1) {
    static std::once_flag attr_once[2];
    cudaError_t attr_err = cudaSuccess;
    std::call_once(attr_once[dtype == RLT_BF16 ? 1 : 0], [&] {
      attr_err = dtype == RLT_BF16
                     ? cudaFuncSetAttribute(paged_prefill_tc_kernel<__nv_bfloat16>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes)
                     : cudaFuncSetAttribute(paged_prefill_tc_kernel<__half>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    });
    if (attr_err != cudaSuccess) return static_cast<int>(attr_err);
    const dim3 grid(static_cast<unsigned>((num_tokens + kTileM - 1) / kTileM + num_seqs), hq);
    if (dtype == RLT_BF16)
      paged_prefill_tc_kernel<__nv_bfloat16><<<grid, kThreads, kSmemBytes, stream>>>(p);
    else
      paged_prefill_tc_kernel<__half><<<grid, kThreads, kSmemBytes, stream>>>(p);
    return launch_status(cudaGetLastError());
  }
  const dim3 grid(static_cast<unsigned>((num_tokens + kPairRows - 1) / kPairRows + num_seqs), hq);
  cudaError_t err;
  if (version == 2)
    err = dtype == RLT_BF16 ? launch_pair<__nv_bfloat16, false, 1>(grid, p, stream)
                            : launch_pair<__half, false, 1>(grid, p, stream);
  else if (version == 3)
    err = dtype == RLT_BF16 ? launch_pair<__nv_bfloat16, true, 1>(grid, p, stream)
                            : launch_pair<__half, true, 1>(grid, p, stream);
  else if (version == 4)
    err = dtype == RLT_BF16 ? launch_pair<__nv_bfloat16, true, 2>(grid, p, stream)
                            : launch_pair<__half, true, 2>(grid, p, stream);
  else if (version == 5)
    err = dtype == RLT_BF16 ? launch_pair<__nv_bfloat16, true, 1, true>(grid, p, stream)
                            : launch_pair<__half, true, 1, true>(grid, p, stream);
  else if (version == 8 && kKeys8 % page == 0)
    err = dtype == RLT_BF16 ? launch_pair8<__nv_bfloat16, true>(grid, p, stream)
                            : launch_pair8<__half, false>(grid, p, stream);
  else  // 6 / 7 (and 8 with 128-token pages): bf16 splits P into hi + lo (fp16's 11-bit P needs no split)
    err = dtype == RLT_BF16 ? launch_pair<__nv_bfloat16, true, 1, true, true>(grid, p, stream)
                            : launch_pair<__half, true, 1, true>(grid, p, stream);
  if (err != cudaSuccess) return static_cast<int>(err);
  return launch_status(cudaGetLastError());
}

}  // namespace detail
}  // namespace rlt

extern "C" int rlt_prefill_tc_select(int32_t version) {
  if (version < 1 || version > 8) return rlt::g_prefill_version.load();
  return rlt::g_prefill_version.exchange(version);
}

extern "C" int rlt_paged_prefill_uses_tensor_cores(int32_t dtype, int32_t head_dim,
                                                   int32_t page_size) {
  return rlt::detail::prefill_tc_shape(dtype, head_dim, page_size) ? 1 : 0;
}
