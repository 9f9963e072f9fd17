// Fused per-layer glue of the Ouro recurrent core (sm_100a):
//  * RMSNorm (optionally with the residual add that follows it),
//  * RoPE on q and k fused with the KV page write into the depth plane,
//  * SwiGLU activation.
// Each reproduces the rounding steps of the reference's torch expressions
// (vllm_rlt/models/ouro.py): every torch op on a 16-bit tensor computes in
// fp32 and rounds its result to the tensor dtype, so the fused kernels round
// at the same points.
#include "common.cuh"

namespace rlt {
namespace {

template <typename T>
__device__ __forceinline__ float rnd(float x) {  // round to T and back (one torch op's output)
  return to_f32<T>(from_f32<T>(x));
}

// One torch elementwise op = one IEEE-rounded fp32 operation (then rounded to
// T): the explicit _rn intrinsics keep the compiler from contracting a
// multiply and an add into one fused multiply-add, which rounds once.
__device__ __forceinline__ float mul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add(float a, float b) { return __fadd_rn(a, b); }

// vllm_rlt/models/ouro.py:33-36:
//   value = x.float(); value = value * rsqrt(mean(value^2) + eps)
//   y = weight * value.to(dtype)            (then, fused: residual + y)
// One CTA per row; the row is cached in registers (hidden <= 32 * 8 * 16).
template <typename T>
__global__ void __launch_bounds__(256) rms_norm_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                       const T* __restrict__ residual, T* __restrict__ out,
                                                       int hidden, float eps, int64_t x_stride,
                                                       int64_t r_stride, int64_t o_stride) {
  const int row = blockIdx.x;
  const T* xr = x + row * x_stride;
  float vals[16];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    vals[i] = c < hidden ? to_f32<T>(xr[c]) : 0.f;
    ss = fmaf(vals[i], vals[i], ss);
  }
  __shared__ float partial[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(kFullMask, ss, o);
  if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? partial[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(kFullMask, t, o);
    if (threadIdx.x == 0) partial[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(partial[0] / static_cast<float>(hidden) + eps);
  T* orow = out + row * o_stride;
  const T* rrow = residual ? residual + row * r_stride : nullptr;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c >= hidden) continue;
    float y = rnd<T>(mul(to_f32<T>(w[c]), rnd<T>(mul(vals[i], inv))));
    if (rrow) y = add(to_f32<T>(rrow[c]), y);
    orow[c] = from_f32<T>(y);
  }
}

// Sum of `v` over the CTA (blockDim a multiple of 32, at most 1024); every
// thread gets the total. `partial` holds 33 floats; it is reused by the next
// call only after the __syncthreads that ends this one.
__device__ __forceinline__ float block_sum(float v, float* partial) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFullMask, v, o);
  if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? partial[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(kFullMask, t, o);
    if (threadIdx.x == 0) partial[32] = t;
  }
  __syncthreads();
  return partial[32];
}

// The same norm on 16-byte vectors (hidden a multiple of the vector width,
// rows 16-byte aligned), each thread holding up to kNV consecutive vectors of
// the row. With w2 set it also writes out2 = RMSNorm(out; w2): the residual
// stream's next norm (ouro.py:118-125, the post-attention norm's output feeds
// the MLP norm; a layer's output feeds the next layer's input norm or the
// final norm), so the pair costs one launch and one read of the row.
template <typename T, int kNV>
__global__ void __launch_bounds__(256) rms_norm_vec_kernel(
    const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ residual,
    T* __restrict__ out, const T* __restrict__ w2, T* __restrict__ out2, int hidden, float eps,
    int64_t x_stride, int64_t r_stride, int64_t o_stride, int64_t o2_stride) {
  constexpr int V = 16 / sizeof(T);
  __shared__ float partial[33];
  const int row = blockIdx.x;
  const int nvec = hidden / V;
  // every input this thread needs is loaded up front (x, the weights, the
  // residual), so the two reductions wait on one memory round trip, not three
  uint4 xr[kNV], wr[kNV], rr[kNV], w2r[kNV];
  const uint4 zero = make_uint4(0, 0, 0, 0);
#pragma unroll
  for (int k = 0; k < kNV; ++k) {
    const int vi = threadIdx.x + k * blockDim.x;
    const bool in = vi < nvec;
    xr[k] = in ? ld_vec(x + row * x_stride + vi * V) : zero;
    wr[k] = in ? ld_vec(w + vi * V) : zero;
    rr[k] = in && residual != nullptr ? ld_vec(residual + row * r_stride + vi * V) : zero;
    w2r[k] = in && w2 != nullptr ? ld_vec(w2 + vi * V) : zero;
  }
  float vals[kNV][V];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kNV; ++k) {
    unpack16<T>(xr[k], vals[k]);
#pragma unroll
    for (int e = 0; e < V; ++e) ss = fmaf(vals[k][e], vals[k][e], ss);
  }
  const float inv = rsqrtf(block_sum(ss, partial) / static_cast<float>(hidden) + eps);
  float ss2 = 0.f;
#pragma unroll
  for (int k = 0; k < kNV; ++k) {
    const int vi = threadIdx.x + k * blockDim.x;
    if (vi >= nvec) continue;
    float wv[V], y[V];
    unpack16<T>(wr[k], wv);
    if (residual != nullptr) {
      float rv[V];
      unpack16<T>(rr[k], rv);
#pragma unroll
      for (int e = 0; e < V; ++e) y[e] = rnd<T>(add(rv[e], rnd<T>(mul(wv[e], rnd<T>(mul(vals[k][e], inv))))));
    } else {
#pragma unroll
      for (int e = 0; e < V; ++e) y[e] = rnd<T>(mul(wv[e], rnd<T>(mul(vals[k][e], inv))));
    }
    st_vec(out + row * o_stride + vi * V, pack16<T>(y));
#pragma unroll
    for (int e = 0; e < V; ++e) {
      vals[k][e] = y[e];
      ss2 = fmaf(y[e], y[e], ss2);
    }
  }
  if (w2 == nullptr) return;  // uniform over the CTA
  const float inv2 = rsqrtf(block_sum(ss2, partial) / static_cast<float>(hidden) + eps);
#pragma unroll
  for (int k = 0; k < kNV; ++k) {
    const int vi = threadIdx.x + k * blockDim.x;
    if (vi >= nvec) continue;
    float wv[V], y[V];
    unpack16<T>(w2r[k], wv);
#pragma unroll
    for (int e = 0; e < V; ++e) y[e] = rnd<T>(mul(wv[e], rnd<T>(mul(vals[k][e], inv2))));
    st_vec(out2 + row * o2_stride + vi * V, pack16<T>(y));
  }
}

// vllm_rlt/models/ouro.py:61-75 and :104-110, fused with the page write of
// vllm_rlt/core/kv_cache_manager.py:531-532:
//   angles = pos.float() * inv_freq  (fp32), cat(angles, angles)
//   cos, sin = angles.cos().to(dtype), angles.sin().to(dtype)
//   q' = q * cos + rotate_half(q) * sin  (each op rounded to dtype), same for k
//   key_cache[block, layer, offset] = k'; value_cache[...] = v
// grid = rows, block = (heads + kv_heads) * head_dim / 2 pairs, capped.
// cos/sin depend only on (row, i): computed once per row into shared memory
// (ouro.py:61-70 computes them once per position too). kVec moves q, k and v
// as 16-byte vectors (every pointer and stride 16-byte aligned, head_dim a
// multiple of two vectors); otherwise element by element.
constexpr int kRopeMaxHalf = 256;  // head_dim <= 512
template <typename T, bool kVec>
__global__ void __launch_bounds__(256) rope_write_kernel(
    const T* __restrict__ qkv, const int64_t* __restrict__ positions,
    const float* __restrict__ inv_freq, T* __restrict__ q_out, T* __restrict__ kc,
    T* __restrict__ vc, const int64_t* __restrict__ blocks, const int64_t* __restrict__ offsets,
    int32_t* status, int heads, int kv_heads, int head_dim, int layer, int page,
    int64_t num_blocks, int64_t qkv_stride, int64_t q_rs, int64_t q_hs, int64_t c_bs,
    int64_t c_ls, int64_t c_ts, int64_t c_hs) {
  __shared__ float cs[2][kRopeMaxHalf];
  const int row = blockIdx.x;
  const int half = head_dim / 2;
  const float pos = static_cast<float>(positions[row]);
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float angle = mul(pos, inv_freq[i]);
    cs[0][i] = rnd<T>(cosf(angle));
    cs[1][i] = rnd<T>(sinf(angle));
  }
  const T* src = qkv + row * qkv_stride;
  const int64_t blk = blocks[row];
  const int64_t off = offsets[row];
  const bool ok = blk >= 0 && blk < num_blocks && off >= 0 && off < page;
  if (!ok && threadIdx.x == 0)
    raise_status(status, (blk < 0 || blk >= num_blocks) ? kStatusBadBlock : kStatusBadOffset);
  const int64_t cache_row = blk * c_bs + layer * c_ls + off * c_ts;
  __syncthreads();
  // first half: x1*cos + (-x2)*sin ; second half: x2*cos + x1*sin
  auto rotate = [&](float x1, float x2, int i, float& y1, float& y2) {
    const float c = cs[0][i], sn = cs[1][i];
    y1 = add(rnd<T>(mul(x1, c)), rnd<T>(mul(-x2, sn)));
    y2 = add(rnd<T>(mul(x2, c)), rnd<T>(mul(x1, sn)));
  };
  if constexpr (kVec) {
    constexpr int V = 16 / sizeof(T);
    const int chunks = half / V;
    const int tasks = (heads + kv_heads) * chunks;
    for (int idx = threadIdx.x; idx < tasks; idx += blockDim.x) {
      const int h = idx / chunks;
      const int i0 = (idx - h * chunks) * V;
      float a[V], b[V], y1[V], y2[V];
      unpack16<T>(ld_vec(src + h * head_dim + i0), a);
      unpack16<T>(ld_vec(src + h * head_dim + i0 + half), b);
#pragma unroll
      for (int e = 0; e < V; ++e) rotate(a[e], b[e], i0 + e, y1[e], y2[e]);
      T* dst;
      if (h < heads)
        dst = q_out + row * q_rs + h * q_hs;
      else if (ok)
        dst = kc + cache_row + (h - heads) * c_hs;
      else
        continue;
      st_vec(dst + i0, pack16<T>(y1));
      st_vec(dst + i0 + half, pack16<T>(y2));
    }
    if (!ok) return;
    const T* vsrc = src + (heads + kv_heads) * head_dim;
    const int vper = head_dim / V;
    for (int idx = threadIdx.x; idx < kv_heads * vper; idx += blockDim.x) {
      const int h = idx / vper;
      const int d = (idx - h * vper) * V;
      st_vec(vc + cache_row + h * c_hs + d, ld_vec(vsrc + h * head_dim + d));
    }
  } else {
    const int rotated = (heads + kv_heads) * half;  // (head, i) pairs that get RoPE
    for (int idx = threadIdx.x; idx < rotated; idx += blockDim.x) {
      const int h = idx / half;
      const int i = idx - h * half;
      float y1, y2;
      rotate(to_f32<T>(src[h * head_dim + i]), to_f32<T>(src[h * head_dim + i + half]), i, y1,
             y2);
      if (h < heads) {
        T* dst = q_out + row * q_rs + h * q_hs;
        dst[i] = from_f32<T>(y1);
        dst[i + half] = from_f32<T>(y2);
      } else if (ok) {
        T* dst = kc + cache_row + (h - heads) * c_hs;
        dst[i] = from_f32<T>(y1);
        dst[i + half] = from_f32<T>(y2);
      }
    }
    if (!ok) return;
    const T* vsrc = src + (heads + kv_heads) * head_dim;
    for (int idx = threadIdx.x; idx < kv_heads * head_dim; idx += blockDim.x) {
      const int h = idx / head_dim;
      const int d = idx - h * head_dim;
      vc[cache_row + h * c_hs + d] = vsrc[idx];
    }
  }
}

// vllm_rlt/models/ouro.py:122-123: silu(gate) * up, each op rounded.
template <typename T>
__global__ void silu_mul_kernel(const T* __restrict__ gu, T* __restrict__ out, int inter,
                                int64_t in_stride, int64_t out_stride, int64_t total) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / inter;
    const int col = static_cast<int>(i - row * inter);
    const float g = to_f32<T>(gu[row * in_stride + col]);
    const float u = to_f32<T>(gu[row * in_stride + inter + col]);
    const float s = rnd<T>(__fdiv_rn(g, add(1.f, expf(-g))));
    out[row * out_stride + col] = from_f32<T>(mul(s, u));
  }
}

// The same on 16-byte vectors (inter a multiple of the vector width, rows
// and pointers 16-byte aligned); the arithmetic per element is unchanged.
template <typename T>
__global__ void silu_mul_vec_kernel(const T* __restrict__ gu, T* __restrict__ out, int inter,
                                    int64_t in_stride, int64_t out_stride, int64_t total_vec) {
  constexpr int V = 16 / sizeof(T);
  const int vpr = inter / V;  // vectors per row
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total_vec;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / vpr;
    const int col = static_cast<int>(i - row * vpr) * V;
    float g[V], u[V], y[V];
    unpack16<T>(ld_vec(gu + row * in_stride + col), g);
    unpack16<T>(ld_vec(gu + row * in_stride + inter + col), u);
#pragma unroll
    for (int e = 0; e < V; ++e) {
      const float sv = rnd<T>(__fdiv_rn(g[e], add(1.f, expf(-g[e]))));
      y[e] = mul(sv, u[e]);
    }
    st_vec(out + row * out_stride + col, pack16<T>(y));
  }
}

int esize(int32_t dtype) { return dtype == RLT_F32 ? 4 : (dtype == RLT_F16 || dtype == RLT_BF16) ? 2 : 0; }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool stride16(int64_t stride, int es) { return (stride * es) % 16 == 0; }

template <typename T>
int launch_rms_norm(const void* x, const void* weight, const void* residual, void* out,
                    const void* weight2, void* out2, int rows, int hidden, float eps,
                    int64_t x_stride, int64_t r_stride, int64_t o_stride, int64_t o2_stride,
                    cudaStream_t s) {
  constexpr int V = 16 / sizeof(T);
  const int es = sizeof(T);
  const bool vec = hidden % V == 0 && aligned16(x) && aligned16(weight) && aligned16(out) &&
                   (residual == nullptr || (aligned16(residual) && stride16(r_stride, es))) &&
                   (weight2 == nullptr || (aligned16(weight2) && aligned16(out2) &&
                                           stride16(o2_stride, es))) &&
                   stride16(x_stride, es) && stride16(o_stride, es);
  const T* xp = static_cast<const T*>(x);
  const T* wp = static_cast<const T*>(weight);
  const T* rp = static_cast<const T*>(residual);
  T* op = static_cast<T*>(out);
  if (vec) {
    const int nvec = hidden / V;
    const int threads = nvec >= 256 ? 256 : (nvec + 31) / 32 * 32;
    const int per = (nvec + threads - 1) / threads;
    const T* w2p = static_cast<const T*>(weight2);
    T* o2p = static_cast<T*>(out2);
#define RLT_NORM_VEC(NV)                                                                    \
  rms_norm_vec_kernel<T, NV><<<rows, threads, 0, s>>>(xp, wp, rp, op, w2p, o2p, hidden, eps, \
                                                      x_stride, r_stride, o_stride, o2_stride)
    if (per == 1)
      RLT_NORM_VEC(1);
    else if (per == 2)
      RLT_NORM_VEC(2);
    else if (per <= 4)
      RLT_NORM_VEC(4);
    else
      return RLT_E_SHAPE;
#undef RLT_NORM_VEC
    return launch_status(cudaGetLastError());
  }
  if (weight2 != nullptr) return RLT_E_ALIGN;  // the fused pair needs the vector layout
  const int threads = hidden >= 2048 ? 256 : 128;
  if (hidden > threads * 16) return RLT_E_SHAPE;
  rms_norm_kernel<T><<<rows, threads, 0, s>>>(xp, wp, rp, op, hidden, eps, x_stride, r_stride,
                                              o_stride);
  return launch_status(cudaGetLastError());
}

int rms_norm_entry(const void* x, const void* weight, const void* residual, void* out,
                   const void* weight2, void* out2, int32_t dtype, int32_t rows, int32_t hidden,
                   float eps, int64_t x_stride, int64_t residual_stride, int64_t out_stride,
                   int64_t out2_stride, void* stream) {
  if (esize(dtype) == 0) return RLT_E_DTYPE;
  if (rows < 0 || hidden <= 0 || hidden > 16 * 256) return RLT_E_SHAPE;
  if ((weight2 == nullptr) != (out2 == nullptr)) return RLT_E_SHAPE;
  if (rows == 0) return RLT_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case RLT_F32:
      return launch_rms_norm<float>(x, weight, residual, out, weight2, out2, rows, hidden, eps,
                                    x_stride, residual_stride, out_stride, out2_stride, s);
    case RLT_F16:
      return launch_rms_norm<__half>(x, weight, residual, out, weight2, out2, rows, hidden, eps,
                                     x_stride, residual_stride, out_stride, out2_stride, s);
    default:
      return launch_rms_norm<__nv_bfloat16>(x, weight, residual, out, weight2, out2, rows,
                                            hidden, eps, x_stride, residual_stride, out_stride,
                                            out2_stride, s);
  }
}

}  // namespace
}  // namespace rlt

using namespace rlt;

extern "C" int rlt_rms_norm(const void* x, const void* weight, const void* residual, void* out,
                            int32_t dtype, int32_t rows, int32_t hidden, float eps,
                            int64_t x_stride, int64_t residual_stride, int64_t out_stride,
                            void* stream) {
  return rms_norm_entry(x, weight, residual, out, nullptr, nullptr, dtype, rows, hidden, eps,
                        x_stride, residual_stride, out_stride, 0, stream);
}

extern "C" int rlt_rms_norm2(const void* x, const void* weight, const void* residual, void* out,
                             const void* weight2, void* out2, int32_t dtype, int32_t rows,
                             int32_t hidden, float eps, int64_t x_stride, int64_t residual_stride,
                             int64_t out_stride, int64_t out2_stride, void* stream) {
  return rms_norm_entry(x, weight, residual, out, weight2, out2, dtype, rows, hidden, eps,
                        x_stride, residual_stride, out_stride, out2_stride, stream);
}

extern "C" int rlt_rope_write_kv(const void* qkv, const int64_t* positions, const float* inv_freq,
                                 void* q_out, void* key_cache, void* value_cache,
                                 const int64_t* write_blocks, const int64_t* write_offsets,
                                 int32_t* status, int32_t dtype, int32_t rows, int32_t heads,
                                 int32_t kv_heads, int32_t head_dim, int32_t layer,
                                 int32_t page_size, int64_t num_blocks, int64_t qkv_stride,
                                 int64_t q_row_stride, int64_t q_head_stride,
                                 int64_t cache_block_stride, int64_t cache_layer_stride,
                                 int64_t cache_token_stride, int64_t cache_head_stride,
                                 void* stream) {
  if (esize(dtype) == 0) return RLT_E_DTYPE;
  if (head_dim <= 0 || head_dim % 2 || head_dim / 2 > kRopeMaxHalf) return RLT_E_HEAD_DIM;
  if (heads <= 0 || kv_heads <= 0 || heads % kv_heads) return RLT_E_HEADS;
  if (rows < 0 || layer < 0 || page_size <= 0 || num_blocks < 0) return RLT_E_SHAPE;
  if (rows == 0) return RLT_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int es = esize(dtype);
  const bool vec = head_dim % (2 * (16 / es)) == 0 && aligned16(qkv) && aligned16(q_out) &&
                   aligned16(key_cache) && aligned16(value_cache) && stride16(qkv_stride, es) &&
                   stride16(q_row_stride, es) && stride16(q_head_stride, es) &&
                   stride16(cache_block_stride, es) && stride16(cache_layer_stride, es) &&
                   stride16(cache_token_stride, es) && stride16(cache_head_stride, es);
#define RLT_ROPE_LAUNCH(T)                                                                      \
  if (vec)                                                                                      \
    RLT_ROPE_KERNEL(T, true);                                                                   \
  else                                                                                          \
    RLT_ROPE_KERNEL(T, false)
#define RLT_ROPE_KERNEL(T, VEC)                                                                 \
  rope_write_kernel<T, VEC><<<rows, 256, 0, s>>>(                                               \
      static_cast<const T*>(qkv), positions, inv_freq, static_cast<T*>(q_out),                  \
      static_cast<T*>(key_cache), static_cast<T*>(value_cache), write_blocks, write_offsets,    \
      status, heads, kv_heads, head_dim, layer, page_size, num_blocks, qkv_stride, q_row_stride, \
      q_head_stride, cache_block_stride, cache_layer_stride, cache_token_stride,                \
      cache_head_stride)
  switch (dtype) {
    case RLT_F32: RLT_ROPE_LAUNCH(float); break;
    case RLT_F16: RLT_ROPE_LAUNCH(__half); break;
    default: RLT_ROPE_LAUNCH(__nv_bfloat16); break;
  }
#undef RLT_ROPE_LAUNCH
#undef RLT_ROPE_KERNEL
  return launch_status(cudaGetLastError());
}

extern "C" int rlt_silu_mul(const void* gate_up, void* out, int32_t dtype, int32_t rows,
                            int32_t intermediate, int64_t in_stride, int64_t out_stride,
                            void* stream) {
  if (esize(dtype) == 0) return RLT_E_DTYPE;
  if (rows < 0 || intermediate <= 0) return RLT_E_SHAPE;
  if (rows == 0) return RLT_OK;
  const int64_t total = static_cast<int64_t>(rows) * intermediate;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int es = esize(dtype);
  const int V = 16 / es;
  if (intermediate % V == 0 && aligned16(gate_up) && aligned16(out) && stride16(in_stride, es) &&
      stride16(out_stride, es) && stride16(intermediate, es)) {
    const int64_t total_vec = total / V;
    const int64_t vblocks64 = (total_vec + 255) / 256;
    const unsigned vblocks = static_cast<unsigned>(vblocks64 < 8192 ? vblocks64 : 8192);
    switch (dtype) {
      case RLT_F32: silu_mul_vec_kernel<float><<<vblocks, 256, 0, s>>>(static_cast<const float*>(gate_up), static_cast<float*>(out), intermediate, in_stride, out_stride, total_vec); break;
      case RLT_F16: silu_mul_vec_kernel<__half><<<vblocks, 256, 0, s>>>(static_cast<const __half*>(gate_up), static_cast<__half*>(out), intermediate, in_stride, out_stride, total_vec); break;
      default: silu_mul_vec_kernel<__nv_bfloat16><<<vblocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(gate_up), static_cast<__nv_bfloat16*>(out), intermediate, in_stride, out_stride, total_vec); break;
    }
    return launch_status(cudaGetLastError());
  }
  const int64_t blocks64 = (total + 255) / 256;
  const unsigned blocks = static_cast<unsigned>(blocks64 < 8192 ? blocks64 : 8192);
  switch (dtype) {
    case RLT_F32: silu_mul_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(gate_up), static_cast<float*>(out), intermediate, in_stride, out_stride, total); break;
    case RLT_F16: silu_mul_kernel<__half><<<blocks, 256, 0, s>>>(static_cast<const __half*>(gate_up), static_cast<__half*>(out), intermediate, in_stride, out_stride, total); break;
    default: silu_mul_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(gate_up), static_cast<__nv_bfloat16*>(out), intermediate, in_stride, out_stride, total); break;
  }
  return launch_status(cudaGetLastError());
}
