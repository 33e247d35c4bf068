// Host runtime of the library: status strings, CUDA error plumbing, and the TMA
// tensor maps that describe a KV pool (built once per pool and cached).
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace pkv {

int num_sms() {
  static int n = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
  });
  return n;
}

namespace {
thread_local std::string g_last_cuda_error;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

struct MapEntry {
  pkv_pool pool;
  int heads_per_box, chunks_per_box;
  CUtensorMap k, v;
};
std::mutex g_map_mutex;
std::vector<MapEntry> g_maps;  // small LRU-free cache: a process holds few pools

bool same_pool(const pkv_pool& a, const pkv_pool& b) { return std::memcmp(&a, &b, sizeof(pkv_pool)) == 0; }
}  // namespace

void set_last_cuda_error(cudaError_t e) { g_last_cuda_error = cudaGetErrorString(e); }

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return PKV_OK;
  set_last_cuda_error(e);
  return PKV_ERR_CUDA;
}

int make_pool_tensor_map(CUtensorMap* map, const void* base, const pkv_pool& pool, int heads_per_box,
                         int chunks_per_box) {
  auto fn = encode_fn();
  if (!fn) {
    g_last_cuda_error = "cuTensorMapEncodeTiled is not available from the driver";
    return PKV_ERR_CUDA;
  }
  const int d = pool.head_dim, bs = pool.block_size;
  const cuuint64_t esz = 2;
  cuuint64_t dims[5] = {64, (cuuint64_t)bs, (cuuint64_t)(d / 64), (cuuint64_t)pool.num_kv_heads,
                        (cuuint64_t)pool.num_layers * (cuuint64_t)pool.num_blocks_total};
  cuuint64_t strides[4] = {(cuuint64_t)d * esz, 64 * esz, (cuuint64_t)bs * d * esz,
                           (cuuint64_t)pool.num_kv_heads * bs * d * esz};
  const cuuint32_t chunks = chunks_per_box > 0 ? (cuuint32_t)chunks_per_box : (cuuint32_t)(d / 64);
  cuuint32_t box[5] = {64, (cuuint32_t)bs, chunks, (cuuint32_t)heads_per_box, 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  const CUtensorMapDataType dt =
      pool.dtype == PKV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, dt, 5, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    g_last_cuda_error = "cuTensorMapEncodeTiled failed with CUresult " + std::to_string((int)r);
    return PKV_ERR_CUDA;
  }
  return PKV_OK;
}

int make_matrix_tensor_map(CUtensorMap* map, const void* base, int dtype, uint64_t inner, uint64_t rows,
                           uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) {
    g_last_cuda_error = "cuTensorMapEncodeTiled is not available from the driver";
    return PKV_ERR_CUDA;
  }
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = dtype == PKV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    g_last_cuda_error = "cuTensorMapEncodeTiled failed with CUresult " + std::to_string((int)r);
    return PKV_ERR_CUDA;
  }
  return PKV_OK;
}

bool get_pool_maps(const pkv_pool& pool, CUtensorMap* tk, CUtensorMap* tv, int heads_per_box, int chunks_per_box) {
  std::lock_guard<std::mutex> lock(g_map_mutex);
  for (const MapEntry& e : g_maps) {
    if (same_pool(e.pool, pool) && e.heads_per_box == heads_per_box && e.chunks_per_box == chunks_per_box) {
      *tk = e.k;
      *tv = e.v;
      return true;
    }
  }
  MapEntry e;
  std::memset(&e, 0, sizeof(e));
  e.pool = pool;
  e.heads_per_box = heads_per_box;
  e.chunks_per_box = chunks_per_box;
  if (make_pool_tensor_map(&e.k, pool.k, pool, heads_per_box, chunks_per_box) != PKV_OK) return false;
  if (make_pool_tensor_map(&e.v, pool.v, pool, heads_per_box, chunks_per_box) != PKV_OK) return false;
  if (g_maps.size() >= 64) g_maps.erase(g_maps.begin());
  g_maps.push_back(e);
  *tk = e.k;
  *tv = e.v;
  return true;
}

}  // namespace pkv

extern "C" const char* pkv_status_string(int status) {
  switch (status) {
    case PKV_OK: return "ok";
    case PKV_ERR_INVALID_ARGUMENT: return "invalid argument";
    case PKV_ERR_OUT_OF_RANGE: return "index out of range";
    case PKV_ERR_WORKSPACE: return "workspace too small";
    case PKV_ERR_CUDA: return "CUDA error";
    case PKV_ERR_NO_BLOCKS: return "not enough free KV cache blocks";
    case PKV_ERR_DOUBLE_FREE: return "slot freed twice";
    case PKV_ERR_UNKNOWN_SLOT: return "unknown slot";
    case PKV_ERR_UNSUPPORTED: return "unsupported shape or dtype";
    case PKV_ERR_TIMEOUT: return "device wait timed out";
    case PKV_ERR_EMPTY_PROMPT: return "prompt is empty";
    case PKV_ERR_PROMPT_TOO_LONG: return "prompt leaves no room to generate (prompt_len >= max_model_len)";
    default: return "unknown status";
  }
}

extern "C" const char* pkv_last_cuda_error(void) { return pkv::g_last_cuda_error.c_str(); }

extern "C" int pkv_version(void) { return 0x000100; }
