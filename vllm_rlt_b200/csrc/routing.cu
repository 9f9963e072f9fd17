// Routing and metadata kernels (sm_100a): depth/page resolution of a routing
// bank, packed-prefill metadata staging and expansion, and resident-slot
// gather/scatter. Integer/byte work, bit-exact with the reference's Triton
// kernels (vllm_rlt/kernels/routing.py, vllm_rlt/kernels/prefill_metadata.py).
#include "common.cuh"

namespace rlt {
namespace {

struct MetadataParams {
  const int64_t* desc;
  const int32_t* tables;
  int64_t* slots;
  int64_t* positions;
  int32_t* lengths;
  int64_t* blocks;
  int64_t* offsets;
  int32_t* out_tables;
  int32_t* status;
  int n, size, width, page, planes, out_width, num_slots;
};

// vllm_rlt/kernels/routing.py:7-41. One CTA per bank row (grid = size).
// Rows >= n are padding: slot = pos = 0, length 0, a zero table row, and no
// write address.
__global__ void __launch_bounds__(256) metadata_kernel(const __grid_constant__ MetadataParams p) {
  const int row = blockIdx.x;
  bool valid = row < p.n;
  int64_t slot = 0, depth = 0, pos = 0;
  if (valid) {
    slot = p.desc[row * 3];
    depth = p.desc[row * 3 + 1];
    pos = p.desc[row * 3 + 2];
  }
  const int64_t plane = p.planes > 1 ? depth : 0;
  const bool in_range = slot >= 0 && slot < p.num_slots && plane >= 0 && plane < p.planes &&
                        pos >= 0 && pos < static_cast<int64_t>(p.width) * p.page;
  if (valid && !in_range) {
    if (threadIdx.x == 0) raise_status(p.status, kStatusBadSlot);
    valid = false;
  }
  const int64_t base = (slot * p.planes + plane) * p.width;
  if (threadIdx.x == 0) {
    p.slots[row] = slot;
    p.positions[row] = pos;
    p.lengths[row] = valid ? static_cast<int32_t>(pos + 1) : 0;
    if (valid) {
      p.blocks[row] = p.tables[base + pos / p.page];
      p.offsets[row] = pos % p.page;
    }
  }
  int32_t* dst = p.out_tables + static_cast<int64_t>(row) * p.width;
  const int32_t* src = p.tables + base;
  for (int col = threadIdx.x; col < p.out_width; col += blockDim.x)
    dst[col] = valid ? src[col] : 0;
}

// vllm_rlt/kernels/prefill_metadata.py:7-12.
__global__ void stage_kernel(const int64_t* __restrict__ src, int64_t* __restrict__ dst,
                             int32_t* __restrict__ dst32, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t v = src[i];
    dst[i] = v;
    dst32[i] = static_cast<int32_t>(v);
  }
}

// vllm_rlt/kernels/prefill_metadata.py:15-32.
__global__ void expand_kernel(const int64_t* __restrict__ positions,
                              const int64_t* __restrict__ sequences,
                              const int32_t* __restrict__ tables, int64_t* __restrict__ blocks,
                              int64_t* __restrict__ offsets, int32_t* status, int64_t n,
                              int width, int page, int64_t entries) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t pos = positions[i];
    const int64_t seq = sequences[i];
    const int64_t idx = seq * width + pos / page;
    if (pos < 0 || seq < 0 || idx >= entries) {
      raise_status(status, kStatusBadSequence);
      continue;
    }
    blocks[i] = tables[idx];
    offsets[i] = pos % page;
  }
}

// vllm_rlt/kernels/routing.py:44-59; grid = (size, column chunks).
template <typename U>
__global__ void gather_kernel(const U* __restrict__ pool, const int64_t* __restrict__ slots,
                              U* __restrict__ out, int n, int width, int64_t in_stride,
                              int64_t out_stride) {
  const int row = blockIdx.x;
  const int col = blockIdx.y * blockDim.x + threadIdx.x;
  if (col >= width) return;
  U value{};
  if (row < n) value = pool[slots[row] * in_stride + col];
  out[row * out_stride + col] = value;
}

// vllm_rlt/kernels/routing.py:62-76; grid = (n, column chunks).
template <typename U>
__global__ void scatter_kernel(const U* __restrict__ values, const int64_t* __restrict__ slots,
                               U* __restrict__ pool, int width, int64_t in_stride,
                               int64_t out_stride) {
  const int row = blockIdx.x;
  const int col = blockIdx.y * blockDim.x + threadIdx.x;
  if (col >= width) return;
  pool[slots[row] * out_stride + col] = values[row * in_stride + col];
}

}  // namespace
}  // namespace rlt

using namespace rlt;

extern "C" int rlt_metadata(const int64_t* descriptor, const int32_t* tables, int64_t* slots,
                            int64_t* positions, int32_t* lengths, int64_t* blocks,
                            int64_t* offsets, int32_t* out_tables, int32_t* status, int32_t n,
                            int32_t size, int32_t width, int32_t page_size, int32_t planes,
                            int32_t out_width, int32_t num_slots, void* stream) {
  if (n < 0 || size < n || width <= 0 || page_size <= 0 || planes <= 0 || out_width < 0 ||
      out_width > width || num_slots <= 0)
    return RLT_E_SHAPE;
  if (size == 0) return RLT_OK;
  MetadataParams p{descriptor, tables, slots,  positions, lengths, blocks,    offsets, out_tables,
                   status,     n,      size,   width,     page_size, planes, out_width, num_slots};
  metadata_kernel<<<size, 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return launch_status(cudaGetLastError());
}

extern "C" int rlt_stage_prefill(const int64_t* source, int64_t* target, int32_t* target32,
                                 int64_t n, void* stream) {
  if (n < 0) return RLT_E_SHAPE;
  if (n == 0) return RLT_OK;
  const int64_t blocks = (n + 255) / 256;
  stage_kernel<<<static_cast<unsigned>(blocks < 4096 ? blocks : 4096), 256, 0,
                 static_cast<cudaStream_t>(stream)>>>(source, target, target32, n);
  return launch_status(cudaGetLastError());
}

extern "C" int rlt_expand_prefill(const int64_t* positions, const int64_t* sequences,
                                  const int32_t* tables, int64_t* blocks, int64_t* offsets,
                                  int32_t* status, int64_t n, int32_t width, int32_t page_size,
                                  int64_t num_table_entries, void* stream) {
  if (n < 0 || width <= 0 || page_size <= 0) return RLT_E_SHAPE;
  if (n == 0) return RLT_OK;
  const int64_t grid = (n + 255) / 256;
  expand_kernel<<<static_cast<unsigned>(grid < 4096 ? grid : 4096), 256, 0,
                  static_cast<cudaStream_t>(stream)>>>(positions, sequences, tables, blocks,
                                                       offsets, status, n, width, page_size,
                                                       num_table_entries);
  return launch_status(cudaGetLastError());
}

extern "C" int rlt_gather(const void* pool, const int64_t* slots, void* out, int32_t n,
                          int32_t size, int32_t width, int32_t elem_bytes, int64_t in_stride,
                          int64_t out_stride, void* stream) {
  if (n < 0 || size < n || width < 0) return RLT_E_SHAPE;
  if (size == 0 || width == 0) return RLT_OK;
  dim3 grid(size, ceil_div(width, 256));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (elem_bytes) {
    case 1: gather_kernel<uint8_t><<<grid, 256, 0, s>>>(static_cast<const uint8_t*>(pool), slots, static_cast<uint8_t*>(out), n, width, in_stride, out_stride); break;
    case 2: gather_kernel<uint16_t><<<grid, 256, 0, s>>>(static_cast<const uint16_t*>(pool), slots, static_cast<uint16_t*>(out), n, width, in_stride, out_stride); break;
    case 4: gather_kernel<uint32_t><<<grid, 256, 0, s>>>(static_cast<const uint32_t*>(pool), slots, static_cast<uint32_t*>(out), n, width, in_stride, out_stride); break;
    case 8: gather_kernel<uint64_t><<<grid, 256, 0, s>>>(static_cast<const uint64_t*>(pool), slots, static_cast<uint64_t*>(out), n, width, in_stride, out_stride); break;
    default: return RLT_E_DTYPE;
  }
  return launch_status(cudaGetLastError());
}

extern "C" int rlt_scatter(const void* values, const int64_t* slots, void* pool, int32_t n,
                           int32_t width, int32_t elem_bytes, int64_t in_stride,
                           int64_t out_stride, void* stream) {
  if (n < 0 || width < 0) return RLT_E_SHAPE;
  if (n == 0 || width == 0) return RLT_OK;
  dim3 grid(n, ceil_div(width, 256));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (elem_bytes) {
    case 1: scatter_kernel<uint8_t><<<grid, 256, 0, s>>>(static_cast<const uint8_t*>(values), slots, static_cast<uint8_t*>(pool), width, in_stride, out_stride); break;
    case 2: scatter_kernel<uint16_t><<<grid, 256, 0, s>>>(static_cast<const uint16_t*>(values), slots, static_cast<uint16_t*>(pool), width, in_stride, out_stride); break;
    case 4: scatter_kernel<uint32_t><<<grid, 256, 0, s>>>(static_cast<const uint32_t*>(values), slots, static_cast<uint32_t*>(pool), width, in_stride, out_stride); break;
    case 8: scatter_kernel<uint64_t><<<grid, 256, 0, s>>>(static_cast<const uint64_t*>(values), slots, static_cast<uint64_t*>(pool), width, in_stride, out_stride); break;
    default: return RLT_E_DTYPE;
  }
  return launch_status(cudaGetLastError());
}
