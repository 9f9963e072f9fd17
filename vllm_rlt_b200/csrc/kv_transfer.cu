// KV page transport for prefill/decode disaggregation: copy byte segments of
// a KV pool into another pool, which may live on another GPU of the node.
//
// The reference moves a request's KV from a prefill worker to a decode worker
// with NIXL one-sided WRITEs of (address, bytes) segments between registered
// pools (vllm_rlt/pd/transport.py:18-176): a fully covered block is one
// segment with all its layers, a partly covered block one segment per layer.
// Here the same segment lists drive one kernel launch per batch: CTA (s, c)
// copies the c-th 64 KiB slice of segment s with 16-byte vector loads and
// stores. A destination on another GPU is written through its peer mapping
// (peer access enabled in this process, or a CUDA-IPC mapping of the other
// process's pool): plain stores over NVLink, no TMA and no multicast.
#include "common.cuh"

namespace rlt {
namespace {

constexpr int kCopyThreads = 256;
constexpr int64_t kSliceBytes = 64 << 10;

__global__ void __launch_bounds__(kCopyThreads) copy_segments_kernel(const int64_t* segments,
                                                                     int32_t* status) {
  const int64_t* d = segments + static_cast<int64_t>(blockIdx.x) * 3;
  const int64_t src = d[0], dst = d[1], bytes = d[2];
  if (((src | dst | bytes) & 15) != 0 || bytes < 0) {
    if (blockIdx.y == 0 && threadIdx.x == 0) raise_status(status, kStatusBadOffset);
    return;
  }
  const int64_t begin = static_cast<int64_t>(blockIdx.y) * kSliceBytes;
  if (begin >= bytes) return;
  const int64_t end = min(bytes, begin + kSliceBytes);
  const char* s = reinterpret_cast<const char*>(src);
  char* t = reinterpret_cast<char*>(dst);
  constexpr int kUnroll = 4;
  int64_t off = begin + static_cast<int64_t>(threadIdx.x) * 16;
  for (; off + (kUnroll - 1) * kCopyThreads * 16 < end; off += kUnroll * kCopyThreads * 16) {
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) v[u] = ld_stream(s + off + u * kCopyThreads * 16);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) st_vec(t + off + u * kCopyThreads * 16, v[u]);
  }
  for (; off < end; off += kCopyThreads * 16) st_vec(t + off, ld_stream(s + off));
}

}  // namespace
}  // namespace rlt

using namespace rlt;

extern "C" int rlt_copy_segments(const int64_t* segments, int32_t num_segments,
                                 int64_t max_segment_bytes, int32_t* status, void* stream) {
  if (num_segments < 0 || max_segment_bytes < 0) return RLT_E_SHAPE;
  if (num_segments == 0 || max_segment_bytes == 0) return RLT_OK;
  if (segments == nullptr) return RLT_E_SHAPE;
  const int64_t slices = (max_segment_bytes + kSliceBytes - 1) / kSliceBytes;
  if (slices > 65535) return RLT_E_SHAPE;
  copy_segments_kernel<<<dim3(num_segments, static_cast<unsigned>(slices)), kCopyThreads, 0,
                         static_cast<cudaStream_t>(stream)>>>(segments, status);
  return launch_status(cudaGetLastError());
}

extern "C" int rlt_enable_peer_access(int32_t peer_device) {
  int current = 0;
  cudaError_t err = cudaGetDevice(&current);
  if (err != cudaSuccess) return static_cast<int>(err);
  if (peer_device == current) return RLT_OK;
  int can = 0;
  err = cudaDeviceCanAccessPeer(&can, current, peer_device);
  if (err != cudaSuccess) return static_cast<int>(err);
  if (!can) return RLT_E_DEVICE;
  err = cudaDeviceEnablePeerAccess(peer_device, 0);
  if (err == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();  // clear the sticky-free error state of this call
    return RLT_OK;
  }
  return launch_status(err);
}
