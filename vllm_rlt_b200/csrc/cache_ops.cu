// KV page write (reshape_and_cache into a depth plane) and the LAST-EXITED
// exit copy, sm_100a. Both are bit-exact byte movers: 16-byte vectors when the
// head rows are 16-byte aligned, element copies otherwise.
#include "common.cuh"

namespace rlt {
namespace {

struct KvWriteParams {
  const char* k;
  const char* v;
  char* kc;
  char* vc;
  const int64_t* blocks;
  const int64_t* offsets;
  int32_t* status;
  int rows, hkv, row_bytes;  // row_bytes = head_dim * esize
  int layer, page;
  int64_t num_blocks;
  // byte strides
  int64_t k_rs, k_hs, v_rs, v_hs, c_bs, c_ls, c_ts, c_hs;
};

// key_cache[blocks[r], layer, offsets[r], h, :] = k[r, h, :] (and V), as
// vllm_rlt/core/kv_cache_manager.py:531-532. One CTA per written row.
template <typename U>
__global__ void __launch_bounds__(128) kv_write_kernel(const __grid_constant__ KvWriteParams p) {
  const int row = blockIdx.x;
  const int64_t blk = p.blocks[row];
  const int64_t off = p.offsets[row];
  if (blk < 0 || blk >= p.num_blocks || off < 0 || off >= p.page) {
    if (threadIdx.x == 0)
      raise_status(p.status, (blk < 0 || blk >= p.num_blocks) ? kStatusBadBlock : kStatusBadOffset);
    return;
  }
  const int64_t dst = blk * p.c_bs + p.layer * p.c_ls + off * p.c_ts;
  const int per_head = p.row_bytes / static_cast<int>(sizeof(U));
  const int total = per_head * p.hkv;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int h = i / per_head;
    const int x = i - h * per_head;
    const int64_t d = dst + h * p.c_hs + x * static_cast<int64_t>(sizeof(U));
    const U kv = *reinterpret_cast<const U*>(p.k + row * p.k_rs + h * p.k_hs + x * sizeof(U));
    const U vv = *reinterpret_cast<const U*>(p.v + row * p.v_rs + h * p.v_hs + x * sizeof(U));
    *reinterpret_cast<U*>(p.kc + d) = kv;
    *reinterpret_cast<U*>(p.vc + d) = vv;
  }
}

struct FinalizeParams {
  const int64_t* desc;
  const int32_t* tables;
  char* kc;
  char* vc;
  int32_t* status;
  int rows, slots, width, planes, page, layers, row_bytes;  // row_bytes = channels * esize
  int64_t num_blocks;
  int64_t bs, ls, ts;  // byte strides of block, layer, token
};

// Exit copy (vllm_rlt/kernels/routing.py:79-109): for descriptor row
// (slot, depth, pos) copy every layer's K/V token row from plane `depth` to
// each plane in (depth, planes). Each 16-byte vector is read once and stored
// to every deeper plane. grid = (rows, chunks of the layers x row vectors).
template <typename U>
__global__ void __launch_bounds__(256) finalize_kernel(const __grid_constant__ FinalizeParams p) {
  const int row = blockIdx.x;
  const int64_t slot = p.desc[row * 3];
  const int64_t depth = p.desc[row * 3 + 1];
  const int64_t pos = p.desc[row * 3 + 2];
  if (slot < 0 || slot >= p.slots || depth < 0 || depth >= p.planes || pos < 0 ||
      pos >= static_cast<int64_t>(p.width) * p.page) {
    if (threadIdx.x == 0 && blockIdx.y == 0) raise_status(p.status, kStatusBadSlot);
    return;
  }
  if (depth + 1 >= p.planes) return;
  const int64_t page_idx = pos / p.page;
  const int64_t off = pos - page_idx * p.page;
  const int32_t* trow = p.tables + slot * p.planes * p.width + page_idx;
  const int64_t src_blk = trow[depth * p.width];
  if (src_blk < 0 || src_blk >= p.num_blocks) {
    if (threadIdx.x == 0 && blockIdx.y == 0) raise_status(p.status, kStatusBadBlock);
    return;
  }
  const int per_layer = p.row_bytes / static_cast<int>(sizeof(U));
  const int total = per_layer * p.layers;
  const int64_t src_base = src_blk * p.bs + off * p.ts;
  for (int i = blockIdx.y * blockDim.x + threadIdx.x; i < total; i += gridDim.y * blockDim.x) {
    const int layer = i / per_layer;
    const int x = i - layer * per_layer;
    const int64_t rel = layer * p.ls + x * static_cast<int64_t>(sizeof(U));
    const U kv = *reinterpret_cast<const U*>(p.kc + src_base + rel);
    const U vv = *reinterpret_cast<const U*>(p.vc + src_base + rel);
    for (int64_t t = depth + 1; t < p.planes; ++t) {
      const int64_t dst_blk = trow[t * p.width];
      if (dst_blk < 0 || dst_blk >= p.num_blocks) {
        raise_status(p.status, kStatusBadBlock);
        continue;
      }
      const int64_t d = dst_blk * p.bs + off * p.ts + rel;
      *reinterpret_cast<U*>(p.kc + d) = kv;
      *reinterpret_cast<U*>(p.vc + d) = vv;
    }
  }
}

int esize_of(int32_t dtype) {
  switch (dtype) {
    case RLT_F32: return 4;
    case RLT_F16:
    case RLT_BF16: return 2;
    default: return 0;
  }
}

bool all16(std::initializer_list<int64_t> values) {
  for (int64_t v : values)
    if (v % 16) return false;
  return true;
}

}  // namespace
}  // namespace rlt

using namespace rlt;

extern "C" int rlt_kv_write(const void* k, const void* v, void* key_cache, void* value_cache,
                            const int64_t* write_blocks, const int64_t* write_offsets,
                            int32_t* status, int32_t dtype, int32_t num_rows,
                            int32_t num_kv_heads, int32_t head_dim, int32_t layer,
                            int32_t page_size, int64_t num_blocks, int64_t k_row_stride,
                            int64_t k_head_stride, int64_t v_row_stride, int64_t v_head_stride,
                            int64_t cache_block_stride, int64_t cache_layer_stride,
                            int64_t cache_token_stride, int64_t cache_head_stride,
                            void* stream) {
  const int es = esize_of(dtype);
  if (es == 0) return RLT_E_DTYPE;
  if (head_dim <= 0) return RLT_E_HEAD_DIM;
  if (num_kv_heads <= 0) return RLT_E_HEADS;
  if (num_rows < 0 || layer < 0 || page_size <= 0 || num_blocks < 0) return RLT_E_SHAPE;
  if (num_rows == 0) return RLT_OK;
  KvWriteParams p{};
  p.k = static_cast<const char*>(k);
  p.v = static_cast<const char*>(v);
  p.kc = static_cast<char*>(key_cache);
  p.vc = static_cast<char*>(value_cache);
  p.blocks = write_blocks;
  p.offsets = write_offsets;
  p.status = status;
  p.rows = num_rows;
  p.hkv = num_kv_heads;
  p.row_bytes = head_dim * es;
  p.layer = layer;
  p.page = page_size;
  p.num_blocks = num_blocks;
  p.k_rs = k_row_stride * es;
  p.k_hs = k_head_stride * es;
  p.v_rs = v_row_stride * es;
  p.v_hs = v_head_stride * es;
  p.c_bs = cache_block_stride * es;
  p.c_ls = cache_layer_stride * es;
  p.c_ts = cache_token_stride * es;
  p.c_hs = cache_head_stride * es;
  const bool vec = all16({reinterpret_cast<int64_t>(k), reinterpret_cast<int64_t>(v),
                          reinterpret_cast<int64_t>(key_cache),
                          reinterpret_cast<int64_t>(value_cache), p.row_bytes, p.k_rs, p.k_hs,
                          p.v_rs, p.v_hs, p.c_bs, p.c_ls, p.c_ts, p.c_hs});
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (vec)
    kv_write_kernel<uint4><<<num_rows, 128, 0, s>>>(p);
  else if (es == 4)
    kv_write_kernel<uint32_t><<<num_rows, 128, 0, s>>>(p);
  else
    kv_write_kernel<uint16_t><<<num_rows, 128, 0, s>>>(p);
  return launch_status(cudaGetLastError());
}

extern "C" int rlt_finalize(const int64_t* descriptor, const int32_t* tables, void* key_cache,
                            void* value_cache, int32_t* status, int32_t dtype, int32_t num_rows,
                            int32_t num_slots, int32_t width, int32_t planes, int32_t page_size,
                            int32_t num_layers, int32_t channels, int64_t num_blocks,
                            int64_t block_stride, int64_t layer_stride, int64_t token_stride,
                            void* stream) {
  const int es = esize_of(dtype);
  if (es == 0) return RLT_E_DTYPE;
  if (num_rows < 0 || num_slots <= 0 || width <= 0 || planes <= 0 || page_size <= 0 ||
      num_layers <= 0 || channels <= 0 || num_blocks < 0)
    return RLT_E_SHAPE;
  if (num_rows == 0 || planes == 1) return RLT_OK;
  FinalizeParams p{};
  p.desc = descriptor;
  p.tables = tables;
  p.kc = static_cast<char*>(key_cache);
  p.vc = static_cast<char*>(value_cache);
  p.status = status;
  p.rows = num_rows;
  p.slots = num_slots;
  p.width = width;
  p.planes = planes;
  p.page = page_size;
  p.layers = num_layers;
  p.row_bytes = channels * es;
  p.num_blocks = num_blocks;
  p.bs = block_stride * es;
  p.ls = layer_stride * es;
  p.ts = token_stride * es;
  const bool vec = all16({reinterpret_cast<int64_t>(key_cache),
                          reinterpret_cast<int64_t>(value_cache), p.row_bytes, p.bs, p.ls, p.ts});
  const int unit = vec ? 16 : es;
  const int total = p.row_bytes / unit * num_layers;
  const int chunks = ceil_div(total, 256 * 4);  // each thread moves up to 4 units
  dim3 grid(num_rows, chunks < 1 ? 1 : chunks);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (vec)
    finalize_kernel<uint4><<<grid, 256, 0, s>>>(p);
  else if (es == 4)
    finalize_kernel<uint32_t><<<grid, 256, 0, s>>>(p);
  else
    finalize_kernel<uint16_t><<<grid, 256, 0, s>>>(p);
  return launch_status(cudaGetLastError());
}
