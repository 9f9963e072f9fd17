// Depth-aware paged decode attention for sm_100a.
//
// Semantics (vllm_rlt/kernels/paged_attention.py:12-36, the reference's torch
// oracle, and the Triton kernel vllm_rlt/kernels/triton_attention.py:13-97):
// every row r has one query token, its own block table (the caller already
// picked the row's depth plane) and a context length len_r; for query head h
//   out[r, h] = softmax_t(q[r, h] . K[t, h / group] * scale) . V[t, h / group]
// over t < len_r, K[t] = key_cache[table[r, t / page], t % page]. fp32 math,
// output in the input dtype, len_r = 0 gives zeros.
//
// Mapping (HBM-bound: every K/V byte is read exactly once per kv head):
//  * grid.x = row x (tasks of the row / warps per CTA), grid.y = split;
//  * a warp task is one kv head with GC query heads of its GQA group, over
//    one split (a contiguous token range) of the row;
//  * LPT = head_dim / (16 B / elt) lanes read one token's 16-byte-aligned
//    head row with one 16-byte load each, so a warp-wide load covers
//    32 / LPT whole token rows (fully used 32-byte sectors);
//  * every lane accumulates dot-product partials for TOK tokens, then a
//    butterfly reduce-scatter (TOK - 1 shuffles) leaves each lane holding the
//    full score of one token; online softmax runs per warp iteration;
//  * probabilities go through a per-warp shared buffer so that each lane can
//    apply them to its own slice of the V rows it loaded;
//  * long rows are split; each split writes an fp32 (acc, max, sum) partial
//    and the last split CTA of a (row, head block) to finish -- counted with
//    an atomic per (row, head block) -- merges them, so there is no separate
//    combine launch. The split plan is a function of the row's own length
//    only, so results are batch-invariant.
#include <atomic>

#include "common.cuh"

namespace rlt {
namespace {

// Tunables (compile-time; the defaults are the measured best on B200).
#ifndef RLT_DECODE_WARPS
#define RLT_DECODE_WARPS 4
#endif
#ifndef RLT_DECODE_MIN_BLOCKS
#define RLT_DECODE_MIN_BLOCKS 4
#endif
#ifndef RLT_DECODE_V_EARLY
#define RLT_DECODE_V_EARLY 1
#endif
#ifndef RLT_DECODE_SPLIT_CHUNK
#define RLT_DECODE_SPLIT_CHUNK 256
#endif
#ifndef RLT_DECODE_TOK_CAP
#define RLT_DECODE_TOK_CAP 8
#endif
#ifndef RLT_DECODE_LPT
#define RLT_DECODE_LPT 1
#endif
constexpr int kDecodeWarps = RLT_DECODE_WARPS;       // warps (= warp tasks) per CTA
constexpr int kSplitAlign = 32;                      // every split starts at a multiple of this
constexpr int kSplitChunk = RLT_DECODE_SPLIT_CHUNK;  // target tokens per split
constexpr int kMaxSplits = 128;                      // cap; longer rows get longer splits
// Polls (128 ns apart) before a CTA waiting for a split-partial ring slot
// gives up: about a second, far beyond any real wait.
constexpr int64_t kRingWaitLimit = int64_t(1) << 23;

struct DecodeParams {
  const void* q;
  const void* k;
  const void* v;
  const int32_t* tables;
  const int32_t* lengths;
  const int32_t* table_index;  // optional row -> table row map (packed prefill); NULL = identity
  void* out;
  float* ws_o;   // [rows, launch_splits, hq, head_dim] unnormalised acc
  float* ws_ml;  // [rows, launch_splits, hq, 2] (running max in log2 units, sum)
  int* counters;  // [rows, hq] finished-split counts (zeroed by the schedule kernel)
  const int* schedule;  // split launches: [rows + 1] first work item of each position of
                        // `order` (NULL: one item per CTA, blockIdx = (row, head block),
                        // split)
  int* work;            // split launches: next unclaimed work item
  // Split partials live in a ring of `ring` slots, one slot per (row, split)
  // of a row that splits: pair j = part_base[row] + split uses slot j % ring
  // once slot_seq[j % ring] == j, and the row's last merge hands each of its
  // slots on (slot_seq += ring). Pairs are claimed in row order and a row's
  // pairs never exceed the ring, so a pair only ever waits for rows whose
  // work items are all claimed by running CTAs.
  const int* order;      // [rows]: the rows in scheduling order (most splits first)
  const int* part_base;  // [rows]: first ring pair of the row (rows with one split: unused)
  int* row_merges;       // [rows]: head blocks of the row merged so far
  int* slot_seq;         // [ring]: the pair each slot accepts next
  int* ring_wraps;       // set by the schedule: this call's pairs exceed the ring
  int ring;
  float* lse;     // optional [rows, hq]: base-2 log-sum-exp of the scaled scores
                  // (max + log2(sum)); -inf for an empty row. NULL: not written
  int32_t* status;
  int rows, hq, hkv, group, head_dim, page, width, launch_splits;
  int64_t num_blocks;
  int64_t q_rs, q_hs, k_bs, k_ts, k_hs, v_bs, v_ts, v_hs, t_rs, o_rs, o_hs;
  float scale_log2;  // softmax scale * log2(e): scores are kept in base 2
};

struct SplitPlan {
  int count;  // number of non-empty splits
  int per;    // tokens per split (multiple of kSplitAlign)
};

// For decode, a function of the row's own length only: the cap `max_splits`
// is the launch's split count, derived from the table width so that it is at
// least min(ceil(len / chunk), kMaxSplits) for every row the table can hold.
// Every row's reduction order is therefore batch-invariant. The packed-prefill
// path launches a single split (max_splits = 1).
__host__ __device__ __forceinline__ SplitPlan split_plan(int ctx, int max_splits) {
  if (ctx <= 0) return {0, 0};
  int n = (ctx + kSplitChunk - 1) / kSplitChunk;
  if (n > kMaxSplits) n = kMaxSplits;
  if (n > max_splits) n = max_splits;
  int per = (ctx + n - 1) / n;
  per = (per + kSplitAlign - 1) / kSplitAlign * kSplitAlign;
  return {(ctx + per - 1) / per, per};
}

__host__ __device__ __forceinline__ int launch_splits_for(int64_t max_ctx) {
  if (max_ctx <= 0) return 1;
  int64_t n = (max_ctx + kSplitChunk - 1) / kSplitChunk;
  return n > kMaxSplits ? kMaxSplits : static_cast<int>(n);
}

// Tokens each lane group covers per warp iteration: as many as the lanes of
// a token row (so a full reduce-scatter ends with one token per lane), capped
// so that TOK partials for GC query heads stay in registers.
__host__ __device__ constexpr int tokens_per_group(int lpt, int gc) {
  return lpt < RLT_DECODE_TOK_CAP / gc ? lpt : RLT_DECODE_TOK_CAP / gc;
}

template <int N>
struct Log2 {
  static constexpr int value = 1 + Log2<N / 2>::value;
};
template <>
struct Log2<1> {
  static constexpr int value = 0;
};

// Length of row `row`, clamped to what its table can address.
__device__ __forceinline__ int checked_length(const DecodeParams& p, int row, bool report) {
  int ctx = p.lengths[row];
  if (ctx < 0 || static_cast<int64_t>(ctx) > static_cast<int64_t>(p.width) * p.page) {
    if (report) raise_status(p.status, kStatusBadLength);
    return 0;
  }
  return ctx;
}

// Merge the split partials of one query head of one row (one warp): the
// splits' base-2 running maxima and sums give each split's weight; the output
// is the weighted sum of the unnormalised accumulators over the total sum.
//
// A row's splits occupy consecutive ring slots starting at part_base[row],
// wrapping past the ring's end at most once, so their partials are two runs
// with a constant stride; the loops walk each run by a plain stride. (Forming
// every split's slot with a modulo, or with a wrap test, inside the loop over
// splits made the merge -- on the critical path of each row's last split --
// cost the whole decode call 6-10 %.)
template <typename T>
__device__ __forceinline__ void merge_splits(const DecodeParams& p, int row, int qh, int count,
                                             int lane) {
  const int first = p.part_base[row] % p.ring;
  const int n1 = min(count, p.ring - first);  // splits before the wrap
  const int64_t stride = p.hq;                // partial rows between consecutive slots
  const int64_t run1 = static_cast<int64_t>(first) * p.hq + qh;  // split 0
  const int64_t run2 = qh - static_cast<int64_t>(n1) * p.hq;     // split n1 at slot 0
  auto at = [&](int sp) { return (sp < n1 ? run1 : run2) + sp * stride; };
  float mx = -INFINITY;
  for (int sp = lane; sp < count; sp += 32) mx = fmaxf(mx, p.ws_ml[at(sp) * 2]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, o));
  const float mref = mx == -INFINITY ? 0.f : mx;
  // each split's weight 2^(m - mref) once, for the whole warp to read below
  __shared__ float weights[kDecodeWarps][kMaxSplits];
  float* w_of = weights[threadIdx.x >> 5];
  float total = 0.f;
  for (int sp = lane; sp < count; sp += 32) {
    const float2 ml = *reinterpret_cast<const float2*>(p.ws_ml + at(sp) * 2);
    const float w = ex2(ml.x - mref);
    w_of[sp] = w;
    total += ml.y * w;
  }
  __syncwarp();
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(kFullMask, total, o);
  const float inv = 1.f / fmaxf(total, 1e-30f);
  if (p.lse != nullptr && lane == 0)
    p.lse[static_cast<int64_t>(row) * p.hq + qh] = mx == -INFINITY ? -INFINITY : mref + __log2f(total);
  T* out = static_cast<T*>(p.out) + row * p.o_rs + qh * p.o_hs;
  for (int d4 = lane; d4 < p.head_dim / 4; d4 += 32) {
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    // splits in order (the sum is the same as one split at a time); unrolled
    // so several partial loads are in flight: a row split 128 ways is merged
    // at the end of the call, on its critical path
    auto accumulate = [&](int64_t base, int s0, int s1) {
#pragma unroll 4
      for (int sp = s0; sp < s1; ++sp) {
        const int64_t r = base + sp * stride;
        const float w = w_of[sp];
        const float4 v = *reinterpret_cast<const float4*>(p.ws_o + r * p.head_dim + d4 * 4);
        a.x = fmaf(v.x, w, a.x);
        a.y = fmaf(v.y, w, a.y);
        a.z = fmaf(v.z, w, a.z);
        a.w = fmaf(v.w, w, a.w);
      }
    };
    accumulate(run1, 0, n1);
    accumulate(run2, n1, count);
    T* dst = out + d4 * 4;
    dst[0] = from_f32<T>(a.x * inv);
    dst[1] = from_f32<T>(a.y * inv);
    dst[2] = from_f32<T>(a.z * inv);
    dst[3] = from_f32<T>(a.w * inv);
  }
}

// One work item: head block `rblock` of row `row`, split `split`.
template <typename T, int D, int GC, bool ALIGNED>
__device__ __forceinline__ void decode_item(const DecodeParams& p, const int row, const int rblock,
                                            const int split) {
  constexpr int VEC = Vec16<T>::kElems;
  constexpr int LPT = D / VEC;  // lanes per token row
  static_assert(LPT >= 4 && LPT <= 32 && (LPT & (LPT - 1)) == 0, "unsupported head_dim");
  constexpr int GROUPS = 32 / LPT;       // token rows per warp-wide load
  constexpr int TOK = tokens_per_group(LPT, GC);  // tokens per lane group per iteration
  constexpr int ITOK = GROUPS * TOK;     // tokens per warp iteration
  constexpr int RS = Log2<TOK>::value;   // reduce-scatter steps
  constexpr int PLAIN = Log2<LPT / TOK>::value;  // remaining plain reduction steps
  static_assert(kSplitAlign % ITOK == 0, "split alignment must cover a warp iteration");

  __shared__ __align__(16) float pbuf[kDecodeWarps][GC][ITOK];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qchunks = p.group / GC;
  const int tasks_per_row = p.hkv * qchunks;
  const int task = rblock * kDecodeWarps + warp;
  // Warps past the row's last task stay alive for the CTA barrier of the
  // split merge; they compute nothing.
  const bool active = task < tasks_per_row;
  const int kvh = (active ? task : 0) / qchunks;
  const int qh0 = kvh * p.group + ((active ? task : 0) - kvh * qchunks) * GC;

  const int g = lane / LPT;  // lane group: which token row of a warp-wide load
  const int s = lane % LPT;  // 16-byte slice of the head row
  T* out = static_cast<T*>(p.out);

  const int ctx = checked_length(p, row, split == 0 && task == 0 && lane == 0);
  if (ctx == 0) {
    if (active && split == 0 && g == 0) {
      const float zero[VEC] = {};
#pragma unroll
      for (int c = 0; c < GC; ++c)
        st_vec(out + row * p.o_rs + (qh0 + c) * p.o_hs + s * VEC, pack16<T>(zero));
    }
    if (p.lse != nullptr && active && split == 0 && lane == 0) {
#pragma unroll
      for (int c = 0; c < GC; ++c) p.lse[static_cast<int64_t>(row) * p.hq + qh0 + c] = -INFINITY;
    }
    return;
  }
  const SplitPlan plan = split_plan(ctx, p.launch_splits);
  if (split >= plan.count) return;
  const int start = split * plan.per;
  const int end = min(ctx, start + plan.per);

  // Query slice, pre-scaled into base-2 logits.
  float qf[GC][VEC];
#pragma unroll
  for (int c = 0; c < GC; ++c) {
    const T* qp = static_cast<const T*>(p.q) + row * p.q_rs + (qh0 + c) * p.q_hs + s * VEC;
    unpack16<T>(ld_vec(qp), qf[c]);
#pragma unroll
    for (int e = 0; e < VEC; ++e) qf[c][e] *= p.scale_log2;
  }

  float acc[GC][VEC];
  float m[GC], lsum[GC];
#pragma unroll
  for (int c = 0; c < GC; ++c) {
    m[c] = -INFINITY;
    lsum[c] = 0.f;
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[c][e] = 0.f;
  }

  const T* kbase = static_cast<const T*>(p.k) + kvh * p.k_hs + s * VEC;
  const T* vbase = static_cast<const T*>(p.v) + kvh * p.v_hs + s * VEC;
  const int32_t* trow = p.tables + (p.table_index ? p.table_index[row] : row) * p.t_rs;
  const int tl = s >> PLAIN;  // token (within the group) whose score this lane ends with
  const bool writer = (s & ((1 << PLAIN) - 1)) == 0;
  const uint4 zero4 = make_uint4(0, 0, 0, 0);

  const int loop_end = active ? end : start;  // idle warps skip the stream
  for (int base = start; base < loop_end; base += ITOK) {
    const int t0 = base + g * TOK;  // first token of this lane group
    uint4 kr[TOK];
    bool page_ok = false;
    int64_t kp = 0, vp = 0;  // aligned path: element offsets of token t0's page row
    int64_t my_k = -1, my_v = 0;  // generic path: offsets of token t0 + s (lane s < TOK)
    if constexpr (ALIGNED) {
      // page % TOK == 0 and t0 % TOK == 0: the group's TOK tokens share a page.
      if (t0 < end) {
        const int blk = __ldg(trow + t0 / p.page);
        if (blk >= 0 && blk < p.num_blocks) {
          const int off = t0 % p.page;
          kp = blk * p.k_bs + off * p.k_ts;
          vp = blk * p.v_bs + off * p.v_ts;
          page_ok = true;
        } else if (s == 0) {
          raise_status(p.status, kStatusBadBlock);
        }
      }
#pragma unroll
      for (int j = 0; j < TOK; ++j)
        kr[j] = (page_ok && t0 + j < end) ? ld_stream(kbase + kp + j * p.k_ts) : zero4;
    } else {
      if (s < TOK) {
        const int t = t0 + s;
        if (t < end) {
          const int blk = __ldg(trow + t / p.page);
          if (blk >= 0 && blk < p.num_blocks) {
            my_k = blk * p.k_bs + (t % p.page) * p.k_ts;
            my_v = blk * p.v_bs + (t % p.page) * p.v_ts;
          } else {
            raise_status(p.status, kStatusBadBlock);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < TOK; ++j) {
        const int64_t kj = __shfl_sync(kFullMask, my_k, g * LPT + j);
        kr[j] = kj >= 0 ? ld_stream(kbase + kj) : zero4;
      }
    }

    // Dot-product partials over this lane's VEC dims for each of TOK tokens.
    float part[GC][TOK];
#pragma unroll
    for (int j = 0; j < TOK; ++j) {
      float kf[VEC];
      unpack16<T>(kr[j], kf);
#pragma unroll
      for (int c = 0; c < GC; ++c) {
        float a = 0.f;
#pragma unroll
        for (int e = 0; e < VEC; ++e) a = fmaf(qf[c][e], kf[e], a);
        part[c][j] = a;
      }
    }

#if RLT_DECODE_V_EARLY
    // Issue the V loads now so they overlap the reductions below.
    uint4 vr[TOK];
    if constexpr (ALIGNED) {
#pragma unroll
      for (int j = 0; j < TOK; ++j)
        vr[j] = (page_ok && t0 + j < end) ? ld_stream(vbase + vp + j * p.v_ts) : zero4;
    } else {
#pragma unroll
      for (int j = 0; j < TOK; ++j) {
        const int64_t kj = __shfl_sync(kFullMask, my_k, g * LPT + j);
        const int64_t vj = __shfl_sync(kFullMask, my_v, g * LPT + j);
        vr[j] = kj >= 0 ? ld_stream(vbase + vj) : zero4;
      }
    }

#endif
    // Butterfly reduce-scatter across the LPT lanes of the group: after step
    // k each lane keeps half of its partials, so lane s ends with token s>>PLAIN.
#pragma unroll
    for (int c = 0; c < GC; ++c) {
#pragma unroll
      for (int step = 0; step < RS; ++step) {
        const int n = TOK >> step;
        const int mask = LPT >> (step + 1);
        const bool upper = (lane & mask) != 0;
#pragma unroll
        for (int j = 0; j < n / 2; ++j) {
          const float send = upper ? part[c][j] : part[c][j + n / 2];
          const float keep = upper ? part[c][j + n / 2] : part[c][j];
          part[c][j] = keep + __shfl_xor_sync(kFullMask, send, mask);
        }
      }
#pragma unroll
      for (int step = 0; step < PLAIN; ++step) {
        const int mask = (LPT / TOK) >> (step + 1);
        part[c][0] += __shfl_xor_sync(kFullMask, part[c][0], mask);
      }
    }

    bool valid;
    if constexpr (ALIGNED) {
      valid = page_ok && (t0 + tl) < end;
    } else {
      valid = __shfl_sync(kFullMask, my_k, g * LPT + tl) >= 0;
    }

#if !RLT_DECODE_V_EARLY
    // Issue the V loads after the reductions (lower register pressure).
    uint4 vr[TOK];
    if constexpr (ALIGNED) {
#pragma unroll
      for (int j = 0; j < TOK; ++j)
        vr[j] = (page_ok && t0 + j < end) ? ld_stream(vbase + vp + j * p.v_ts) : zero4;
    } else {
#pragma unroll
      for (int j = 0; j < TOK; ++j) {
        const int64_t kj = __shfl_sync(kFullMask, my_k, g * LPT + j);
        const int64_t vj = __shfl_sync(kFullMask, my_v, g * LPT + j);
        vr[j] = kj >= 0 ? ld_stream(vbase + vj) : zero4;
      }
    }

#endif
    // Online softmax (base 2) over the warp's ITOK tokens.
#pragma unroll
    for (int c = 0; c < GC; ++c) {
      const float sc = valid ? part[c][0] : -INFINITY;
      float mt = sc;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(kFullMask, mt, o));
      const float mnew = fmaxf(m[c], mt);
      const float mref = mnew == -INFINITY ? 0.f : mnew;
      const float corr = ex2(m[c] - mref);
      const float pr = ex2(sc - mref);
      m[c] = mnew;
      lsum[c] = lsum[c] * corr + (writer ? pr : 0.f);
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc[c][e] *= corr;
      if (writer) pbuf[warp][c][g * TOK + tl] = pr;
    }
    __syncwarp();

#pragma unroll
    for (int c = 0; c < GC; ++c) {
      float pj[TOK];
#pragma unroll
      for (int j = 0; j < TOK; j += 4) {
        const float4 w = *reinterpret_cast<const float4*>(&pbuf[warp][c][g * TOK + j]);
        pj[j] = w.x;
        pj[j + 1] = w.y;
        pj[j + 2] = w.z;
        pj[j + 3] = w.w;
      }
#pragma unroll
      for (int j = 0; j < TOK; ++j) {
        float vf[VEC];
        unpack16<T>(vr[j], vf);
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[c][e] = fmaf(pj[j], vf[e], acc[c][e]);
      }
    }
    __syncwarp();
  }

  // Merge the lane groups (they covered different tokens of the same dims).
#pragma unroll
  for (int c = 0; c < GC; ++c) {
#pragma unroll
    for (int o = LPT; o < 32; o <<= 1) {
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc[c][e] += __shfl_xor_sync(kFullMask, acc[c][e], o);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lsum[c] += __shfl_xor_sync(kFullMask, lsum[c], o);
  }

  if (plan.count == 1) {
    if (active && g == 0) {
#pragma unroll
      for (int c = 0; c < GC; ++c) {
        const float inv = 1.f / fmaxf(lsum[c], 1e-30f);
        float o[VEC];
#pragma unroll
        for (int e = 0; e < VEC; ++e) o[e] = acc[c][e] * inv;
        st_vec(out + row * p.o_rs + (qh0 + c) * p.o_hs + s * VEC, pack16<T>(o));
      }
    }
    if (p.lse != nullptr && active && lane == 0) {
#pragma unroll
      for (int c = 0; c < GC; ++c)
        p.lse[static_cast<int64_t>(row) * p.hq + qh0 + c] = m[c] + __log2f(lsum[c]);
    }
    return;
  }
  // The ring slot of this (row, split) must have been handed on by the row
  // that used it before (bounded wait; on time-out the call is flagged).
  const int pair = p.part_base[row] + split;
  const bool wraps = *p.ring_wraps != 0;  // uniform over the launch
  if (wraps) {
    if (threadIdx.x == 0) {
      const int* seq = p.slot_seq + pair % p.ring;
      for (int64_t spins = 0; ld_acquire_gpu(seq) != pair; ++spins) {
        if (spins > kRingWaitLimit) {
          raise_status(p.status, kStatusTimeout);
          break;
        }
        __nanosleep(128);
      }
    }
    __syncthreads();
  }
  const int64_t slot = static_cast<int64_t>(pair % p.ring) * p.hq + qh0;
  if (active && g == 0) {
#pragma unroll
    for (int c = 0; c < GC; ++c) {
      float* dst = p.ws_o + (slot + c) * p.head_dim + s * VEC;
#pragma unroll
      for (int e = 0; e < VEC; e += 4)
        *reinterpret_cast<float4*>(dst + e) =
            make_float4(acc[c][e], acc[c][e + 1], acc[c][e + 2], acc[c][e + 3]);
    }
  }
  if (active && lane == 0) {
#pragma unroll
    for (int c = 0; c < GC; ++c)
      *reinterpret_cast<float2*>(p.ws_ml + (slot + c) * 2) = make_float2(m[c], lsum[c]);
  }
  // The last split CTA of this (row, head block) to finish merges them all
  // (no separate combine launch). Partials are made visible before counting.
  __threadfence();
  __syncthreads();
  __shared__ int merge_here;
  if (threadIdx.x == 0) {
    const int done = atomicAdd(p.counters + static_cast<int64_t>(row) * p.hq + rblock, 1);
    merge_here = done == plan.count - 1;
  }
  __syncthreads();
  if (!merge_here) return;
  __threadfence();
  if (active) {
#pragma unroll
    for (int c = 0; c < GC; ++c) merge_splits<T>(p, row, qh0 + c, plan.count, lane);
  }
  // The row's last head block to merge hands its ring slots on (only when
  // this call's pairs wrap around the ring; otherwise no slot is reused).
  if (!wraps) return;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int tasks_per_row = p.hkv * (p.group / GC);
    const int blocks_per_row = (tasks_per_row + kDecodeWarps - 1) / kDecodeWarps;
    if (atomicAdd(p.row_merges + row, 1) == blocks_per_row - 1) {
      for (int sp = 0; sp < plan.count; ++sp)
        st_release_gpu(p.slot_seq + (p.part_base[row] + sp) % p.ring,
                       p.part_base[row] + sp + p.ring);
    }
  }
}

// Split launches run a fixed grid (one resident wave) whose CTAs claim work
// items -- (row, split, head block), row-major, only splits that hold tokens
// -- from a counter, after decode_schedule_kernel has laid the items out.
// Launching one CTA per (row, head block, possible split) instead left most
// CTAs with nothing to do on short rows, and their launches delayed the long
// rows' splits. Single-split launches keep one CTA per (row, head block).
template <typename T, int D, int GC, bool ALIGNED>
__global__ void __launch_bounds__(kDecodeWarps * 32, RLT_DECODE_MIN_BLOCKS)
    paged_decode_kernel(const __grid_constant__ DecodeParams p) {
  const int tasks_per_row = p.hkv * (p.group / GC);
  const int blocks_per_row = (tasks_per_row + kDecodeWarps - 1) / kDecodeWarps;
  if (p.schedule == nullptr) {
    const int row = blockIdx.x / blocks_per_row;
    decode_item<T, D, GC, ALIGNED>(p, row, blockIdx.x - row * blocks_per_row, blockIdx.y);
    return;
  }
  __shared__ int claimed;
  const int total = p.schedule[p.rows];
  for (;;) {
    if (threadIdx.x == 0) claimed = atomicAdd(p.work, 1);
    __syncthreads();
    const int item = claimed;
    __syncthreads();  // every thread has read it before thread 0 claims the next
    if (item >= total) break;
    int lo = 0, hi = p.rows - 1;  // the position: last q with schedule[q] <= item
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.schedule[mid] <= item) lo = mid; else hi = mid - 1;
    }
    const int local = item - p.schedule[lo];
    decode_item<T, D, GC, ALIGNED>(p, p.order[lo], local % blocks_per_row,
                                   local / blocks_per_row);
  }
}

// Work items of a split launch. Rows are taken longest first (by split
// count; the order among rows with equal counts is whatever the placement
// atomics give, which changes no result: a (row, split) partial and the
// merge order do not depend on when or where they run), so the longest rows'
// splits start in the first wave and short rows fill the tail. Position q of
// that order is row order[q]; it gets (its split count, 1 for an empty or
// invalid row) x head blocks items starting at schedule[q], schedule[rows] =
// total, and its splits take ring pairs part_base[order[q]] onwards. Also
// clears the merge, claim and row-merge counters and the ring. One CTA.
constexpr int kScheduleThreads = 1024;

__device__ __forceinline__ int scheduled_splits(const DecodeParams& p, int r) {
  const int len = p.lengths[r];
  const bool ok = len > 0 && static_cast<int64_t>(len) <= static_cast<int64_t>(p.width) * p.page;
  return ok ? split_plan(len, p.launch_splits).count : 1;
}

__global__ void __launch_bounds__(kScheduleThreads) decode_schedule_kernel(
    const __grid_constant__ DecodeParams p, int blocks_per_row, int* counters, int* schedule,
    int* work) {
  constexpr int kScheduleWarps = kScheduleThreads / 32;
  static_assert(kScheduleWarps <= 32, "warp totals scanned by one warp");
  __shared__ int wsum[kScheduleWarps], wpsum[kScheduleWarps];  // per-warp inclusive totals
  __shared__ int bucket[kMaxSplits + 1];  // rows per split count, then placement cursors
  // one pass (rows <= kScheduleThreads): the scan reads the order and the
  // split counts from here instead of a global round trip
  __shared__ int s_order[kScheduleThreads], s_splits[kScheduleThreads];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool one_pass = p.rows <= kScheduleThreads;
  const int my_splits = one_pass && tid < p.rows ? scheduled_splits(p, tid) : 0;
  const int64_t ncounters = static_cast<int64_t>(p.rows) * p.hq;
  for (int64_t i = tid; i < ncounters; i += kScheduleThreads) counters[i] = 0;
  for (int i = tid; i < p.rows; i += kScheduleThreads) p.row_merges[i] = 0;
  for (int i = tid; i < p.ring; i += kScheduleThreads) p.slot_seq[i] = i;
  for (int i = tid; i <= kMaxSplits; i += kScheduleThreads) bucket[i] = 0;
  if (tid == 0) *work = 0;
  __syncthreads();
  if (one_pass) {
    if (tid < p.rows) atomicAdd(&bucket[my_splits], 1);
  } else {
    for (int r = tid; r < p.rows; r += kScheduleThreads) atomicAdd(&bucket[scheduled_splits(p, r)], 1);
  }
  __syncthreads();
  if (warp == 0) {  // first position of each split count, most splits first
    // lane l holds counts kMaxSplits - 5 l ... kMaxSplits - 5 l - 4
    constexpr int kPer = (kMaxSplits + 1 + 31) / 32;
    int n[kPer], sum = 0;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int c = kMaxSplits - (lane * kPer + i);
      n[i] = c >= 0 ? bucket[c] : 0;
      sum += n[i];
    }
    int incl = sum;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int y = __shfl_up_sync(kFullMask, incl, off);
      if (lane >= off) incl += y;
    }
    int at = incl - sum;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int c = kMaxSplits - (lane * kPer + i);
      if (c >= 0) bucket[c] = at;
      at += n[i];
    }
  }
  __syncthreads();
  int* order = const_cast<int*>(p.order);
  if (one_pass) {
    if (tid < p.rows) {
      const int at = RLT_DECODE_LPT ? atomicAdd(&bucket[my_splits], 1) : tid;
      order[at] = tid;
      s_order[at] = tid;
      s_splits[at] = my_splits;
    }
  } else {
    for (int r = tid; r < p.rows; r += kScheduleThreads)
      order[RLT_DECODE_LPT ? atomicAdd(&bucket[scheduled_splits(p, r)], 1) : r] = r;
  }
  __syncthreads();  // the order is visible to the whole CTA
  int carry = 0, pcarry = 0;
  int* part_base = const_cast<int*>(p.part_base);
  for (int base = 0; base < p.rows; base += kScheduleThreads) {
    const int q = base + tid;
    int items = 0, pairs = 0, r = 0;
    if (q < p.rows) {
      r = one_pass ? s_order[q] : order[q];
      const int count = one_pass ? s_splits[q] : scheduled_splits(p, r);
      items = count * blocks_per_row;
      pairs = count > 1 ? count : 0;  // rows with one split write no partials
    }
    // inclusive scans of (items, pairs): within each warp by shuffles, then
    // over the warp totals by warp 0
    int a = items, b = pairs;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int ya = __shfl_up_sync(kFullMask, a, off);
      const int yb = __shfl_up_sync(kFullMask, b, off);
      if (lane >= off) {
        a += ya;
        b += yb;
      }
    }
    if (lane == 31) {
      wsum[warp] = a;
      wpsum[warp] = b;
    }
    __syncthreads();
    if (warp == 0) {
      int x = lane < kScheduleWarps ? wsum[lane] : 0;
      int y = lane < kScheduleWarps ? wpsum[lane] : 0;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int ux = __shfl_up_sync(kFullMask, x, off);
        const int uy = __shfl_up_sync(kFullMask, y, off);
        if (lane >= off) {
          x += ux;
          y += uy;
        }
      }
      if (lane < kScheduleWarps) {
        wsum[lane] = x;
        wpsum[lane] = y;
      }
    }
    __syncthreads();
    if (warp > 0) {
      a += wsum[warp - 1];
      b += wpsum[warp - 1];
    }
    if (q < p.rows) {
      schedule[q] = carry + a - items;
      part_base[r] = pcarry + b - pairs;
    }
    carry += wsum[kScheduleWarps - 1];
    pcarry += wpsum[kScheduleWarps - 1];
    __syncthreads();  // the warp totals are rewritten by the next rows
  }
  if (tid == 0) {
    schedule[p.rows] = carry;
    *p.ring_wraps = pcarry > p.ring;
  }
}

// Any head_dim <= 256, any alignment: one warp per (row, query head), dims
// spread over lanes, tokens in order. Used when the fast kernel's 16-byte
// vector contract does not hold (odd head_dim, unaligned strides).
template <typename T>
__global__ void __launch_bounds__(128) paged_decode_generic_kernel(const __grid_constant__ DecodeParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = static_cast<int64_t>(blockIdx.x) * 4 + (threadIdx.x >> 5);
  if (wid >= static_cast<int64_t>(p.rows) * p.hq) return;
  const int row = static_cast<int>(wid / p.hq);
  const int qh = static_cast<int>(wid % p.hq);
  const int kvh = qh / p.group;
  const int D = p.head_dim;
  const int ctx = checked_length(p, row, qh == 0 && lane == 0);
  const T* qp = static_cast<const T*>(p.q) + row * p.q_rs + qh * p.q_hs;
  float qv[8], acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int d = lane + 32 * i;
    qv[i] = d < D ? to_f32<T>(qp[d]) * p.scale_log2 : 0.f;
    acc[i] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const int32_t* trow = p.tables + (p.table_index ? p.table_index[row] : row) * p.t_rs;
  for (int t = 0; t < ctx; ++t) {
    const int blk = __ldg(trow + t / p.page);
    if (blk < 0 || blk >= p.num_blocks) {
      if (lane == 0) raise_status(p.status, kStatusBadBlock);
      continue;
    }
    const T* kp = static_cast<const T*>(p.k) + blk * p.k_bs + (t % p.page) * p.k_ts + kvh * p.k_hs;
    const T* vp = static_cast<const T*>(p.v) + blk * p.v_bs + (t % p.page) * p.v_ts + kvh * p.v_hs;
    float part = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int d = lane + 32 * i;
      if (d < D) part = fmaf(qv[i], to_f32<T>(kp[d]), part);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(kFullMask, part, o);
    const float mnew = fmaxf(m, part);
    const float corr = ex2(m - mnew);
    const float pr = ex2(part - mnew);
    l = l * corr + pr;
    m = mnew;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int d = lane + 32 * i;
      acc[i] = fmaf(pr, d < D ? to_f32<T>(vp[d]) : 0.f, acc[i] * corr);
    }
  }
  T* op = static_cast<T*>(p.out) + row * p.o_rs + qh * p.o_hs;
  const float inv = 1.f / fmaxf(l, 1e-30f);
  if (p.lse != nullptr && lane == 0)
    p.lse[static_cast<int64_t>(row) * p.hq + qh] = l > 0.f ? m + __log2f(l) : -INFINITY;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int d = lane + 32 * i;
    if (d < D) op[d] = from_f32<T>(acc[i] * inv);
  }
}

// Packed chunked prefill as decode rows (vllm_rlt/kernels/flash_attention.py:
// 66-96 semantics): token i of sequence s (cu[s] <= i < cu[s+1]) reads table
// row s with the bottom-right causal length len_s - qlen_s + (i - cu[s]) + 1.
__global__ void prefill_rows_kernel(const int32_t* __restrict__ cu, const int32_t* __restrict__ lengths,
                                    int32_t* __restrict__ row_seq, int32_t* __restrict__ row_len,
                                    int32_t* status, int num_tokens, int num_seqs) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= num_tokens) return;
  // last s with cu[s] <= i
  int lo = 0, hi = num_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= i) lo = mid; else hi = mid - 1;
  }
  const int begin = cu[lo], stop = cu[lo + 1];
  if (i < begin || i >= stop) {
    raise_status(status, kStatusBadSequence);
    row_seq[i] = 0;
    row_len[i] = 0;
    return;
  }
  const int len = lengths[lo] - (stop - begin) + (i - begin) + 1;
  row_seq[i] = lo;
  row_len[i] = len > 0 ? len : 0;
}

// SM count of the current device (cached per device).
int sm_count() {
  static std::atomic<int> cache[64];
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return 148;
  int n = cache[device].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
      n = 148;
    cache[device].store(n, std::memory_order_relaxed);
  }
  return n;
}

template <typename T, int D, int GC>
cudaError_t launch_fast(const DecodeParams& p, cudaStream_t stream) {
  constexpr int VEC = Vec16<T>::kElems;
  constexpr int LPT = D / VEC;
  constexpr int TOK = tokens_per_group(LPT, GC);
  const int tasks = p.hkv * (p.group / GC);
  const int blocks_per_row = (tasks + kDecodeWarps - 1) / kDecodeWarps;
  dim3 grid(static_cast<unsigned>(p.rows) * blocks_per_row, p.launch_splits);
  if (p.schedule != nullptr) {
    decode_schedule_kernel<<<1, kScheduleThreads, 0, stream>>>(
        p, blocks_per_row, p.counters, const_cast<int*>(p.schedule), p.work);
    const int64_t most = static_cast<int64_t>(p.rows) * blocks_per_row * p.launch_splits;
    const int64_t wave = static_cast<int64_t>(sm_count()) * RLT_DECODE_MIN_BLOCKS;
    grid = dim3(static_cast<unsigned>(most < wave ? most : wave), 1);
  }
  if (p.page % TOK == 0)
    paged_decode_kernel<T, D, GC, true><<<grid, kDecodeWarps * 32, 0, stream>>>(p);
  else
    paged_decode_kernel<T, D, GC, false><<<grid, kDecodeWarps * 32, 0, stream>>>(p);
  return cudaGetLastError();
}

template <typename T, int D>
cudaError_t launch_gc(const DecodeParams& p, cudaStream_t stream) {
  if (p.group % 2 == 0) return launch_fast<T, D, 2>(p, stream);
  return launch_fast<T, D, 1>(p, stream);
}

template <typename T>
cudaError_t launch_typed(DecodeParams p, bool fast, cudaStream_t stream) {
  if (fast) {
    switch (p.head_dim) {
      case 32: return launch_gc<T, 32>(p, stream);
      case 64: return launch_gc<T, 64>(p, stream);
      case 128: return launch_gc<T, 128>(p, stream);
      case 256:
        if constexpr (sizeof(T) == 2) return launch_gc<T, 256>(p, stream);
        break;
      default: break;
    }
  }
  p.launch_splits = 1;  // the generic kernel never splits
  const int64_t warps = static_cast<int64_t>(p.rows) * p.hq;
  paged_decode_generic_kernel<T><<<static_cast<unsigned>((warps + 3) / 4), 128, 0, stream>>>(p);
  return cudaGetLastError();
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

int elem_size(int32_t dtype) {
  switch (dtype) {
    case RLT_F32: return 4;
    case RLT_F16:
    case RLT_BF16: return 2;
    default: return 0;
  }
}

// Whether the 16-byte vector kernel applies to this head_dim / dtype.
bool fast_head_dim(int head_dim, int esize) {
  if (esize == 2) return head_dim == 32 || head_dim == 64 || head_dim == 128 || head_dim == 256;
  return head_dim == 32 || head_dim == 64 || head_dim == 128;
}

}  // namespace
}  // namespace rlt

using namespace rlt;

extern "C" int rlt_version(void) { return 100; }

namespace {

struct DecodeArgs {
  const void* q;
  const void* k;
  const void* v;
  const int32_t* tables;
  int32_t* status;
  int32_t dtype, rows, hq, hkv, head_dim, page, width;
  int64_t num_blocks, q_rs, q_hs, k_bs, k_ts, k_hs, v_bs, v_ts, v_hs, t_rs, o_rs, o_hs;
  void* out;
  float scale;
};

size_t align16(size_t n) { return (n + 15) & ~static_cast<size_t>(15); }

// Ring slots of split partials: one per (row, split) the launch can produce
// when that is few, else enough for the in-flight window -- at least two
// rows' worth of splits (a row never waits for itself) and kRingMin.
constexpr int kRingMin = 4096;
int ring_slots(int rows, int splits) {
  const int64_t most = static_cast<int64_t>(rows) * splits;
  const int64_t window = 2 * static_cast<int64_t>(splits) > kRingMin ? 2 * splits : kRingMin;
  return static_cast<int>(most < window ? most : window);
}

// Split scratch: [rows * hq] merge counters | [rows + 1] schedule | claim
// counter | [rows] order | [rows] ring base | [rows] row merges | [ring] slot
// sequence | ring wrap flag | acc partials [ring, hq, head_dim] | (max, sum)
// partials [ring, hq, 2].
size_t counter_bytes(int rows, int hq, int ring) {
  return align16((static_cast<size_t>(rows) * hq + 4 * static_cast<size_t>(rows) + 3 + ring) *
                 sizeof(int));
}

size_t split_bytes(int rows, int hq, int head_dim, int page, int width) {
  const int splits = launch_splits_for(static_cast<int64_t>(page) * width);
  if (splits <= 1 || rows <= 0 || hq <= 0 || head_dim <= 0) return 0;
  const int ring = ring_slots(rows, splits);
  return counter_bytes(rows, hq, ring) +
         static_cast<size_t>(ring) * hq * (head_dim + 2) * sizeof(float);
}

int validate(const DecodeArgs& a) {
  if (elem_size(a.dtype) == 0) return RLT_E_DTYPE;
  if (a.head_dim <= 0 || a.head_dim > 256) return RLT_E_HEAD_DIM;
  if (a.hq <= 0 || a.hkv <= 0 || a.hq % a.hkv) return RLT_E_HEADS;
  if (a.rows < 0 || a.page <= 0 || a.width < 0 || a.num_blocks < 0) return RLT_E_SHAPE;
  return RLT_OK;
}

// Fill the kernel parameters and pick the vector or generic kernel.
DecodeParams make_params(const DecodeArgs& a, bool* fast) {
  DecodeParams p{};
  p.q = a.q;
  p.k = a.k;
  p.v = a.v;
  p.tables = a.tables;
  p.out = a.out;
  p.status = a.status;
  p.rows = a.rows;
  p.hq = a.hq;
  p.hkv = a.hkv;
  p.group = a.hq / a.hkv;
  p.head_dim = a.head_dim;
  p.page = a.page;
  p.width = a.width;
  p.num_blocks = a.num_blocks;
  p.q_rs = a.q_rs;
  p.q_hs = a.q_hs;
  p.k_bs = a.k_bs;
  p.k_ts = a.k_ts;
  p.k_hs = a.k_hs;
  p.v_bs = a.v_bs;
  p.v_ts = a.v_ts;
  p.v_hs = a.v_hs;
  p.t_rs = a.t_rs;
  p.o_rs = a.o_rs;
  p.o_hs = a.o_hs;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  // The 16-byte vector contract: every base pointer and every stride that
  // moves between head rows is a multiple of 16 bytes.
  const int esize = elem_size(a.dtype);
  const int64_t vec = 16 / esize;
  bool ok = fast_head_dim(a.head_dim, esize) && aligned16(a.q) && aligned16(a.k) &&
            aligned16(a.v) && aligned16(a.out);
  for (int64_t st : {a.q_rs, a.q_hs, a.k_bs, a.k_ts, a.k_hs, a.v_bs, a.v_ts, a.v_hs, a.o_rs,
                     a.o_hs})
    ok = ok && (st % vec == 0);
  *fast = ok;
  p.launch_splits = ok ? launch_splits_for(static_cast<int64_t>(a.page) * a.width) : 1;
  return p;
}

int run(DecodeParams p, int32_t dtype, bool fast, void* split_ws, cudaStream_t s) {
  if (p.launch_splits > 1) {
    // The merge and claim counters and the work schedule are rebuilt on the
    // stream by decode_schedule_kernel on every call (allocation-free and
    // capturable).
    p.ring = ring_slots(p.rows, p.launch_splits);
    const size_t cbytes = counter_bytes(p.rows, p.hq, p.ring);
    p.counters = static_cast<int*>(split_ws);
    p.schedule = p.counters + static_cast<size_t>(p.rows) * p.hq;
    p.work = const_cast<int*>(p.schedule) + p.rows + 1;
    p.order = p.work + 1;
    p.part_base = p.order + p.rows;
    p.row_merges = const_cast<int*>(p.part_base) + p.rows;
    p.slot_seq = p.row_merges + p.rows;
    p.ring_wraps = p.slot_seq + p.ring;
    p.ws_o = reinterpret_cast<float*>(static_cast<char*>(split_ws) + cbytes);
    p.ws_ml = p.ws_o + static_cast<size_t>(p.ring) * p.hq * p.head_dim;
  }
  cudaError_t err;
  switch (dtype) {
    case RLT_F32: err = launch_typed<float>(p, fast, s); break;
    case RLT_F16: err = launch_typed<__half>(p, fast, s); break;
    default: err = launch_typed<__nv_bfloat16>(p, fast, s); break;
  }
  return launch_status(err);
}

}  // namespace

namespace rlt {
namespace detail {

constexpr int kNotEligible = 1;

// Tensor-core packed prefill (paged_prefill_tc.cu); kNotEligible when the
// shape is outside what it covers.
int paged_prefill_tc(const void* q, const void* key_cache, const void* value_cache,
                     const int32_t* block_tables, const int32_t* context_lengths,
                     const int32_t* cu_seqlens_q, void* out, int32_t* status, int32_t dtype,
                     int32_t num_tokens, int32_t num_seqs, int32_t hq, int32_t hkv,
                     int32_t head_dim, int32_t page, int32_t width, int64_t num_blocks,
                     const int64_t* st, float scale, cudaStream_t stream);

// Decode with caller-provided split scratch of `capacity` bytes (the static
// scratch of the no-allocation entry point). Same kernels, same split plan
// and therefore the same results as rlt_paged_decode.
int paged_decode_into(const void* q, const void* key_cache, const void* value_cache,
                      const int32_t* block_tables, const int32_t* context_lengths, void* out,
                      void* scratch, size_t capacity, int32_t* status, int32_t dtype,
                      int32_t num_rows, int32_t num_q_heads, int32_t num_kv_heads,
                      int32_t head_dim, int32_t page_size, int32_t table_width,
                      int64_t num_blocks, const int64_t* strides, float scale,
                      cudaStream_t stream, size_t* needed) {
  const DecodeArgs a{q, key_cache, value_cache, block_tables, status, dtype, num_rows,
                     num_q_heads, num_kv_heads, head_dim, page_size, table_width, num_blocks,
                     strides[0], strides[1], strides[2], strides[3], strides[4], strides[5],
                     strides[6], strides[7], strides[8], strides[9], strides[10], out, scale};
  const int bad = validate(a);
  if (bad != RLT_OK) return bad;
  if (num_rows == 0) return RLT_OK;
  bool fast = false;
  DecodeParams p = make_params(a, &fast);
  p.lengths = context_lengths;
  *needed = 0;
  if (p.launch_splits > 1) {
    *needed = split_bytes(num_rows, num_q_heads, head_dim, page_size, table_width);
    if (*needed > capacity) return RLT_E_WORKSPACE;
  }
  return run(p, dtype, fast, scratch, stream);
}

}  // namespace detail
}  // namespace rlt

extern "C" size_t rlt_paged_decode_workspace_bytes(int32_t num_rows, int32_t num_q_heads,
                                                   int32_t head_dim, int32_t page_size,
                                                   int32_t table_width) {
  return split_bytes(num_rows, num_q_heads, head_dim, page_size, table_width);
}

namespace {
int paged_decode_entry(const void* q, const void* key_cache, const void* value_cache,
                       const int32_t* block_tables, const int32_t* context_lengths, void* out,
                       void* workspace, size_t workspace_bytes, int32_t* status, int32_t dtype,
                       int32_t num_rows, int32_t num_q_heads, int32_t num_kv_heads,
                       int32_t head_dim, int32_t page_size, int32_t table_width,
                       int64_t num_blocks, int64_t q_row_stride, int64_t q_head_stride,
                       int64_t k_block_stride, int64_t k_token_stride, int64_t k_head_stride,
                       int64_t v_block_stride, int64_t v_token_stride, int64_t v_head_stride,
                       int64_t table_row_stride, int64_t out_row_stride,
                       int64_t out_head_stride, float scale, float* lse, void* stream) {
  const DecodeArgs a{q, key_cache, value_cache, block_tables, status, dtype, num_rows,
                     num_q_heads, num_kv_heads, head_dim, page_size, table_width, num_blocks,
                     q_row_stride, q_head_stride, k_block_stride, k_token_stride, k_head_stride,
                     v_block_stride, v_token_stride, v_head_stride, table_row_stride,
                     out_row_stride, out_head_stride, out, scale};
  const int bad = validate(a);
  if (bad != RLT_OK) return bad;
  if (num_rows == 0) return RLT_OK;
  bool fast = false;
  DecodeParams p = make_params(a, &fast);
  p.lengths = context_lengths;
  p.lse = lse;
  if (p.launch_splits > 1) {
    const size_t need = split_bytes(num_rows, num_q_heads, head_dim, page_size, table_width);
    if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))
      return RLT_E_WORKSPACE;
  }
  return run(p, dtype, fast, workspace, static_cast<cudaStream_t>(stream));
}
}  // namespace

extern "C" int rlt_paged_decode(const void* q, const void* key_cache, const void* value_cache,
                                const int32_t* block_tables, const int32_t* context_lengths,
                                void* out, void* workspace, size_t workspace_bytes,
                                int32_t* status, int32_t dtype, int32_t num_rows,
                                int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                int32_t page_size, int32_t table_width, int64_t num_blocks,
                                int64_t q_row_stride, int64_t q_head_stride,
                                int64_t k_block_stride, int64_t k_token_stride,
                                int64_t k_head_stride, int64_t v_block_stride,
                                int64_t v_token_stride, int64_t v_head_stride,
                                int64_t table_row_stride, int64_t out_row_stride,
                                int64_t out_head_stride, float scale, void* stream) {
  return paged_decode_entry(q, key_cache, value_cache, block_tables, context_lengths, out,
                            workspace, workspace_bytes, status, dtype, num_rows, num_q_heads,
                            num_kv_heads, head_dim, page_size, table_width, num_blocks,
                            q_row_stride, q_head_stride, k_block_stride, k_token_stride,
                            k_head_stride, v_block_stride, v_token_stride, v_head_stride,
                            table_row_stride, out_row_stride, out_head_stride, scale, nullptr,
                            stream);
}

extern "C" int rlt_paged_decode_lse(const void* q, const void* key_cache, const void* value_cache,
                                    const int32_t* block_tables, const int32_t* context_lengths,
                                    void* out, void* workspace, size_t workspace_bytes,
                                    int32_t* status, int32_t dtype, int32_t num_rows,
                                    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                    int32_t page_size, int32_t table_width, int64_t num_blocks,
                                    int64_t q_row_stride, int64_t q_head_stride,
                                    int64_t k_block_stride, int64_t k_token_stride,
                                    int64_t k_head_stride, int64_t v_block_stride,
                                    int64_t v_token_stride, int64_t v_head_stride,
                                    int64_t table_row_stride, int64_t out_row_stride,
                                    int64_t out_head_stride, float scale, float* lse,
                                    void* stream) {
  if (lse == nullptr) return RLT_E_SHAPE;
  return paged_decode_entry(q, key_cache, value_cache, block_tables, context_lengths, out,
                            workspace, workspace_bytes, status, dtype, num_rows, num_q_heads,
                            num_kv_heads, head_dim, page_size, table_width, num_blocks,
                            q_row_stride, q_head_stride, k_block_stride, k_token_stride,
                            k_head_stride, v_block_stride, v_token_stride, v_head_stride,
                            table_row_stride, out_row_stride, out_head_stride, scale, lse,
                            stream);
}

extern "C" size_t rlt_paged_prefill_workspace_bytes(int32_t num_tokens, int32_t num_q_heads,
                                                    int32_t head_dim, int32_t page_size,
                                                    int32_t table_width) {
  (void)num_q_heads;
  (void)head_dim;
  (void)page_size;
  (void)table_width;
  if (num_tokens <= 0) return 0;
  // Per-token (table row, causal length) pairs. The CUDA-core path runs one
  // split per token row (thousands of rows already fill the GPU), so it
  // needs no split partials; the tensor-core path needs no scratch at all.
  return align16(static_cast<size_t>(num_tokens) * 2 * sizeof(int32_t));
}

extern "C" int rlt_paged_prefill(const void* q, const void* key_cache, const void* value_cache,
                                 const int32_t* block_tables, const int32_t* context_lengths,
                                 const int32_t* cu_seqlens_q, void* out, void* workspace,
                                 size_t workspace_bytes, int32_t* status, int32_t dtype,
                                 int32_t num_tokens, int32_t num_seqs, int32_t max_seqlen_q,
                                 int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                 int32_t page_size, int32_t table_width, int64_t num_blocks,
                                 int64_t q_row_stride, int64_t q_head_stride,
                                 int64_t k_block_stride, int64_t k_token_stride,
                                 int64_t k_head_stride, int64_t v_block_stride,
                                 int64_t v_token_stride, int64_t v_head_stride,
                                 int64_t table_row_stride, int64_t out_row_stride,
                                 int64_t out_head_stride, float scale, void* stream) {
  (void)max_seqlen_q;  // the launch shape never depends on host-known lengths
  const int64_t strides[11] = {q_row_stride,     q_head_stride,  k_block_stride, k_token_stride,
                               k_head_stride,    v_block_stride, v_token_stride, v_head_stride,
                               table_row_stride, out_row_stride, out_head_stride};
  const DecodeArgs a{q, key_cache, value_cache, block_tables, status, dtype, num_tokens,
                     num_q_heads, num_kv_heads, head_dim, page_size, table_width, num_blocks,
                     q_row_stride, q_head_stride, k_block_stride, k_token_stride, k_head_stride,
                     v_block_stride, v_token_stride, v_head_stride, table_row_stride,
                     out_row_stride, out_head_stride, out, scale};
  const int bad = validate(a);
  if (bad != RLT_OK) return bad;
  if (num_seqs < 0) return RLT_E_SHAPE;
  if (num_tokens == 0) return RLT_OK;
  if (num_seqs == 0) return RLT_E_SHAPE;
  const size_t need = rlt_paged_prefill_workspace_bytes(num_tokens, num_q_heads, head_dim,
                                                        page_size, table_width);
  if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))
    return RLT_E_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int tc = detail::paged_prefill_tc(q, key_cache, value_cache, block_tables, context_lengths,
                                          cu_seqlens_q, out, status, dtype, num_tokens, num_seqs,
                                          num_q_heads, num_kv_heads, head_dim, page_size,
                                          table_width, num_blocks, strides, scale, s);
  if (tc != detail::kNotEligible) return tc;
  int32_t* row_seq = static_cast<int32_t*>(workspace);
  int32_t* row_len = row_seq + num_tokens;
  prefill_rows_kernel<<<ceil_div(num_tokens, 256), 256, 0, s>>>(
      cu_seqlens_q, context_lengths, row_seq, row_len, status, num_tokens, num_seqs);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return launch_status(err);
  bool fast = false;
  DecodeParams p = make_params(a, &fast);
  p.lengths = row_len;
  p.table_index = row_seq;
  p.launch_splits = 1;
  return run(p, dtype, fast, nullptr, s);
}
