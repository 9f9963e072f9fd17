// Paged decode attention without any device allocation.
//
// Some callers cannot call cudaMalloc (or any allocating library routine) at
// the point where they run attention: a runtime whose device memory is fully
// reserved up front by its own pool, an embedding host that forbids driver
// allocations after start-up, or code running inside a region where an
// allocation would synchronise the device. rlt_paged_decode_noalloc serves
// them: it takes the same inputs and outputs as rlt_paged_decode, but its
// split-KV scratch is the file-scope device array below instead of a
// caller-provided workspace.
//
// The array is a fixed 16 MiB per GPU that loads this part of the library and
// stays allocated until the process exits. The driver places it when the
// library's device code is loaded on a device; under lazy module loading
// (CUDA_MODULE_LOADING=LAZY) that happens at the first call on the device, so
// make that call at start-up. All calls share the array and it keeps the
// previous call's contents: each call's first kernel (the one-CTA split
// schedule, on the call's stream) resets the split counters before the
// decode kernel uses them, and a call reads only split partials it wrote
// itself. Two calls that overlap on the GPU (different streams, or different
// host threads on the same device) race on the array: serialise them.
//
// The device address of the array is looked up once per device and cached
// for the life of the process; this assumes the device is not reset
// (cudaDeviceReset) while the library is in use, since a reset unloads the
// module and the array may come back elsewhere.
#include <mutex>

#include "common.cuh"

namespace rlt {
namespace detail {
int paged_decode_into(const void* q, const void* key_cache, const void* value_cache,
                      const int32_t* block_tables, const int32_t* context_lengths, void* out,
                      void* scratch, size_t capacity, int32_t* status, int32_t dtype,
                      int32_t num_rows, int32_t num_q_heads, int32_t num_kv_heads,
                      int32_t head_dim, int32_t page_size, int32_t table_width,
                      int64_t num_blocks, const int64_t* strides, float scale,
                      cudaStream_t stream, size_t* needed);
}  // namespace detail

namespace {

constexpr size_t kScratchBytes = size_t(16) << 20;  // RLT_NOALLOC_SCRATCH_BYTES
static_assert(kScratchBytes == RLT_NOALLOC_SCRATCH_BYTES, "header and library disagree");

static __device__ __align__(256) unsigned char g_decode_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_lock;
void* g_scratch_address[kMaxDevices] = {};

// Device address of this device's copy of the scratch array. In host code
// `g_decode_scratch` is only a host-side stand-in: its device address has to
// be looked up per device, with that device current.
int scratch_address(void** out) {
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return static_cast<int>(err);
  if (device < 0 || device >= kMaxDevices) return RLT_E_DEVICE;
  std::lock_guard<std::mutex> guard(g_lock);
  if (g_scratch_address[device] == nullptr) {
    void* ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_decode_scratch);
    if (err != cudaSuccess || ptr == nullptr) return err != cudaSuccess ? static_cast<int>(err) : RLT_E_DEVICE;
    g_scratch_address[device] = ptr;
  }
  *out = g_scratch_address[device];
  return RLT_OK;
}

}  // namespace
}  // namespace rlt

using namespace rlt;

extern "C" int rlt_paged_decode_noalloc(
    const void* q, const void* key_cache, const void* value_cache, const int32_t* block_tables,
    const int32_t* context_lengths, void* out, int32_t* status, int32_t dtype, int32_t num_rows,
    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int32_t page_size,
    int32_t table_width, int64_t num_blocks, int64_t q_row_stride, int64_t q_head_stride,
    int64_t k_block_stride, int64_t k_token_stride, int64_t k_head_stride,
    int64_t v_block_stride, int64_t v_token_stride, int64_t v_head_stride,
    int64_t table_row_stride, int64_t out_row_stride, int64_t out_head_stride, float scale,
    void* stream) {
  void* scratch = nullptr;
  const int found = scratch_address(&scratch);
  if (found != RLT_OK) return found;
  const int64_t strides[11] = {q_row_stride,     q_head_stride,  k_block_stride, k_token_stride,
                               k_head_stride,    v_block_stride, v_token_stride, v_head_stride,
                               table_row_stride, out_row_stride, out_head_stride};
  size_t needed = 0;
  const int rc = detail::paged_decode_into(
      q, key_cache, value_cache, block_tables, context_lengths, out, scratch, kScratchBytes,
      status, dtype, num_rows, num_q_heads, num_kv_heads, head_dim, page_size, table_width,
      num_blocks, strides, scale, static_cast<cudaStream_t>(stream), &needed);
  return rc == RLT_E_WORKSPACE ? RLT_E_SCRATCH : rc;
}
