// KV append: scatter new K/V rows into paged blocks through slot_mapping.
//
// Replaces the index_put scatters of the reference,
//   k_layer[write_blocks, :, write_offsets] = k[:, :, 0]      (engine/kv_cache.py:613-614)
//   k_layer[where_0, :, where_2] = k[0].transpose(0, 1)        (engine/kv_cache.py:288-289)
// with slot = block * block_size + offset. One thread moves one 16-byte vector
// of one (token, head) row of both K and V when the inputs allow 16-byte
// accesses, else one 4-byte word. The copy is bit-exact.
#include "common.cuh"

namespace pkv {
namespace {

struct AppendParams {
  const uint8_t* k_new;
  const uint8_t* v_new;
  uint8_t* k_pool;
  uint8_t* v_pool;
  const int64_t* slots;
  int32_t* status;
  int64_t n_tokens, tok_stride_b, head_stride_b;  // strides in bytes
  int64_t layer_base;                             // first block row of this layer
  int32_t hkv, bs, row_bytes, nbt;
};

template <typename V>
__global__ void append_kernel(const AppendParams p) {
  const int per_row = p.row_bytes / (int)sizeof(V);
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = p.n_tokens * p.hkv * per_row;
  if (i >= total) return;
  const int u = (int)(i % per_row);
  const int h = (int)((i / per_row) % p.hkv);
  const int64_t t = i / ((int64_t)per_row * p.hkv);
  const int64_t slot = p.slots[t];
  if (slot < 0) return;
  if (slot >= (int64_t)p.nbt * p.bs) {
    report(p.status, PKV_ERR_OUT_OF_RANGE);
    return;
  }
  const int64_t src = t * p.tok_stride_b + h * p.head_stride_b + (int64_t)u * sizeof(V);
  const int64_t dst = (((p.layer_base + slot / p.bs) * p.hkv + h) * p.bs + slot % p.bs) * p.row_bytes +
                      (int64_t)u * sizeof(V);
  *reinterpret_cast<V*>(p.k_pool + dst) = *reinterpret_cast<const V*>(p.k_new + src);
  *reinterpret_cast<V*>(p.v_pool + dst) = *reinterpret_cast<const V*>(p.v_new + src);
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int pkv_kv_append(const pkv_pool* pool, int32_t layer, const void* k_new, const void* v_new,
                             int64_t n_tokens, int64_t tok_stride, int64_t head_stride, const int64_t* slot_mapping,
                             int32_t* status_dev, pkv_stream_t stream) {
  if (!pool || !k_new || !v_new || !slot_mapping || n_tokens < 0) return PKV_ERR_INVALID_ARGUMENT;
  if (layer < 0 || layer >= pool->num_layers || pool->head_dim <= 0 || (pool->head_dim & 1))
    return PKV_ERR_INVALID_ARGUMENT;
  if (pool->dtype != PKV_F16 && pool->dtype != PKV_BF16) return PKV_ERR_UNSUPPORTED;
  if (n_tokens == 0) return PKV_OK;
  AppendParams p;
  p.k_new = static_cast<const uint8_t*>(k_new);
  p.v_new = static_cast<const uint8_t*>(v_new);
  p.k_pool = static_cast<uint8_t*>(pool->k);
  p.v_pool = static_cast<uint8_t*>(pool->v);
  p.slots = slot_mapping;
  p.status = status_dev;
  p.n_tokens = n_tokens;
  p.tok_stride_b = tok_stride * 2;
  p.head_stride_b = head_stride * 2;
  p.layer_base = (int64_t)layer * pool->num_blocks_total;
  p.hkv = pool->num_kv_heads;
  p.bs = pool->block_size;
  p.row_bytes = pool->head_dim * 2;
  p.nbt = pool->num_blocks_total;
  const uintptr_t bits = reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new) |
                         (uintptr_t)p.tok_stride_b | (uintptr_t)p.head_stride_b | (uintptr_t)p.row_bytes;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int threads = 256;
  if ((bits & 15) == 0) {
    const int64_t total = n_tokens * p.hkv * (p.row_bytes / 16);
    append_kernel<uint4><<<(unsigned)((total + threads - 1) / threads), threads, 0, st>>>(p);
  } else if ((bits & 3) == 0) {
    const int64_t total = n_tokens * p.hkv * (p.row_bytes / 4);
    append_kernel<uint32_t><<<(unsigned)((total + threads - 1) / threads), threads, 0, st>>>(p);
  } else {
    const int64_t total = n_tokens * p.hkv * (p.row_bytes / 2);
    append_kernel<uint16_t><<<(unsigned)((total + threads - 1) / threads), threads, 0, st>>>(p);
  }
  return launch_status();
}
