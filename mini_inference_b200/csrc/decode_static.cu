// Decode attention that allocates nothing: the split-sequence state that
// pkv_decode_attention keeps in a caller workspace lives here in one file-scope
// device array instead.
//
// Who needs it: a caller that reaches this library through a plain C FFI
// (ctypes, cgo, JNI) from a process whose device memory belongs to another
// allocator, e.g. PyTorch's caching allocator. Such a caller has no handle on
// that allocator, and a cudaMalloc/cudaFree of its own in the middle of a decode
// step would bypass the allocator's accounting of free HBM (the KV pool is sized
// from it) and may synchronise the device. This entry point lets it run a decode
// step with no device buffer of its own besides the ones the step already has.
//
// Limits: the scratch is one array per device, shared by every call on that
// device, so calls that overlap on the GPU (two streams, two host threads) race
// on it and must be serialised by the caller. Its size is fixed at build time;
// a call that would need more is refused with PKV_ERR_WORKSPACE. The first call
// on a device does the set-up below (a symbol lookup and one clear of the
// array); make that first call before any stream capture.
#include <mutex>

#include "common.cuh"

namespace pkv {
namespace {

constexpr int64_t kScratchBytes = PKV_DECODE_STATIC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

// Ticket counters first, then the partial softmax states of split items (the layout
// pkv_decode_attention gives a caller workspace).
static __device__ __align__(256) uint8_t g_decode_scratch[kScratchBytes];

std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Address of the current device's scratch. The first call for a device looks it
// up and clears it on `stream`, ahead of the kernel that follows on that stream:
// the ticket counters must start at zero (every call leaves them at zero again).
int device_scratch(void** out, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev < 0 || dev >= kMaxDevices) return PKV_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_ptr[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_decode_scratch);
    if (e != cudaSuccess) return cuda_status(e);
    e = cudaMemsetAsync(ptr, 0, kScratchBytes, stream);
    if (e != cudaSuccess) return cuda_status(e);
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return PKV_OK;
}

}  // namespace
}  // namespace pkv

extern "C" int pkv_decode_static_scratch(void** address, int64_t* bytes, pkv_stream_t stream) {
  if (!address || !bytes) return PKV_ERR_INVALID_ARGUMENT;
  const int st = pkv::device_scratch(address, reinterpret_cast<cudaStream_t>(stream));
  *bytes = st == PKV_OK ? pkv::kScratchBytes : 0;
  return st;
}

extern "C" int pkv_decode_static_reset(pkv_stream_t stream) {
  void* scratch = nullptr;
  const int st = pkv::device_scratch(&scratch, reinterpret_cast<cudaStream_t>(stream));
  if (st != PKV_OK) return st;
  // The ticket counters lead the array, laid out as in a caller workspace.
  return pkv_decode_reset_workspace(scratch, pkv::kScratchBytes, stream);
}

extern "C" int pkv_decode_attention_static(const pkv_pool* pool, int32_t layer, const pkv_tables* tables,
                                           int32_t batch, int32_t num_q_heads, void* out, int64_t out_stride_b,
                                           int64_t out_stride_h, const void* q, int64_t q_stride_b,
                                           int64_t q_stride_h, const void* k_new, const void* v_new,
                                           int64_t kv_stride_b, int64_t kv_stride_h, const int64_t* slot_mapping,
                                           const int32_t* context_lens, float scale, int32_t flags,
                                           int32_t* status_dev, pkv_stream_t stream) {
  void* scratch = nullptr;
  const int st = pkv::device_scratch(&scratch, reinterpret_cast<cudaStream_t>(stream));
  if (st != PKV_OK) return st;
  // The decode launcher checks the scratch against what this launch needs and
  // returns PKV_ERR_WORKSPACE, launching nothing, when the array is too small.
  return pkv_decode_attention(pool, layer, tables, batch, num_q_heads, out, out_stride_b, out_stride_h, q, q_stride_b,
                              q_stride_h, k_new, v_new, kv_stride_b, kv_stride_h, slot_mapping, context_lens, scale,
                              flags, scratch, pkv::kScratchBytes, status_dev, stream);
}
