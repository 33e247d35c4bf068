// Rotary position embedding of the qkv projection's rows, fused with the KV append.
//
// Replaces, per layer and forward, the split and head views of Attention.forward, the
// table lookup of RotaryEmbedding.forward and apply_rope on q and k
// (engine/model.py:201-224, 236-249), and -- when slot_mapping is given -- the index_put
// append of the new K/V rows (engine/kv_cache.py:288-289, 613-614): one launch instead
// of the reference's eight elementwise launches and the scatter, reading each qkv row
// once. The rotation repeats the reference's eager arithmetic operation by operation:
//   out = r(r(x * cos) + r(rotate_half(x) * sin)),  rotate_half(x) = cat(-x2, x1)
// where r() rounds to the storage dtype and each product and the sum are computed in
// float32 (the products exactly), so q and k come out bit-identical to the reference's
// on the same cos/sin tables. The tables are inputs: the reference's fp32 tables cast to
// the storage dtype, built by the same torch calls (ops.rope_tables).
//
// One CTA per token; a thread rotates EW consecutive elements of the first half of a
// head together with their partners d/2 further (16-byte accesses when every pointer
// and stride allows, else 4-byte), or copies EW elements of a V row into the pool.
#include "common.cuh"

namespace pkv {
namespace {

struct RopeParams {
  const void* qkv;
  const int64_t* positions;
  const void* cos;
  const void* sin;
  void* q_out;
  void* k_out;
  void* k_pool;
  void* v_pool;
  const int64_t* slots;
  int32_t* status;
  int64_t qkv_stride, q_st, q_sh, k_st, k_sh, max_positions, layer_base;
  int32_t hq, hkv, d, bs, nbt;
};

template <typename T, int EW> struct alignas(EW * sizeof(T)) Pack {
  T v[EW];
};

template <typename T, int EW>
__device__ inline Pack<T, EW> ld(const T* p) {
  return *reinterpret_cast<const Pack<T, EW>*>(p);
}
template <typename T, int EW>
__device__ inline void st(T* p, const Pack<T, EW>& x) {
  *reinterpret_cast<Pack<T, EW>*>(p) = x;
}

// r(r(x * c) + r(y * s)) elementwise, as the reference's eager ops round.
template <typename T, int EW>
__device__ inline Pack<T, EW> rotate(const Pack<T, EW>& x, const Pack<T, EW>& c, const Pack<T, EW>& y,
                                     const Pack<T, EW>& s) {
  Pack<T, EW> out;
#pragma unroll
  for (int e = 0; e < EW; ++e) {
    const T a = Dt<T>::from_f(Dt<T>::to_f(x.v[e]) * Dt<T>::to_f(c.v[e]));
    const T b = Dt<T>::from_f(Dt<T>::to_f(y.v[e]) * Dt<T>::to_f(s.v[e]));
    out.v[e] = Dt<T>::from_f(Dt<T>::to_f(a) + Dt<T>::to_f(b));
  }
  return out;
}

template <typename T, int EW>
__device__ inline Pack<T, EW> negate(const Pack<T, EW>& x) {
  Pack<T, EW> out;
#pragma unroll
  for (int e = 0; e < EW; ++e) out.v[e] = Dt<T>::from_f(-Dt<T>::to_f(x.v[e]));  // exact
  return out;
}

template <typename T, int EW>
__global__ void rope_append_kernel(const RopeParams p) {
  const int64_t t = blockIdx.x;
  const int d = p.d, half = d / 2, per_half = half / EW;
  const int rot_units = (p.hq + p.hkv) * per_half;
  int64_t pos = p.positions[t];
  if (pos < 0 || pos >= p.max_positions) {
    if (threadIdx.x == 0) report(p.status, PKV_ERR_OUT_OF_RANGE);
    pos = 0;  // the status word fails the call; keep the accesses in bounds
  }
  int64_t slot = p.slots ? p.slots[t] : -1;
  if (slot >= (int64_t)p.nbt * p.bs) {
    if (threadIdx.x == 0) report(p.status, PKV_ERR_OUT_OF_RANGE);
    slot = -1;
  }
  const int v_units = slot >= 0 ? p.hkv * (d / EW) : 0;
  const T* row = static_cast<const T*>(p.qkv) + t * p.qkv_stride;
  const T* crow = static_cast<const T*>(p.cos) + pos * d;
  const T* srow = static_cast<const T*>(p.sin) + pos * d;
  for (int u = threadIdx.x; u < rot_units + v_units; u += blockDim.x) {
    if (u < rot_units) {
      const int head = u / per_half, c = (u % per_half) * EW;
      const T* src = row + head * d;
      const Pack<T, EW> x1 = ld<T, EW>(src + c), x2 = ld<T, EW>(src + c + half);
      // rotate_half: element i < d/2 pairs with -x[i + d/2], element i + d/2 with x[i].
      const Pack<T, EW> y1 = rotate<T, EW>(x1, ld<T, EW>(crow + c), negate<T, EW>(x2), ld<T, EW>(srow + c));
      const Pack<T, EW> y2 = rotate<T, EW>(x2, ld<T, EW>(crow + c + half), x1, ld<T, EW>(srow + c + half));
      if (head < p.hq) {
        T* dst = static_cast<T*>(p.q_out) + t * p.q_st + head * p.q_sh;
        st<T, EW>(dst + c, y1);
        st<T, EW>(dst + c + half, y2);
      } else {
        const int kh = head - p.hq;
        if (p.k_out) {
          T* dst = static_cast<T*>(p.k_out) + t * p.k_st + kh * p.k_sh;
          st<T, EW>(dst + c, y1);
          st<T, EW>(dst + c + half, y2);
        }
        if (slot >= 0) {
          T* dst = static_cast<T*>(p.k_pool) + ((p.layer_base + slot / p.bs) * p.hkv + kh) * p.bs * d + (slot % p.bs) * d;
          st<T, EW>(dst + c, y1);
          st<T, EW>(dst + c + half, y2);
        }
      }
    } else {  // V rows go to the pool unchanged
      const int w = u - rot_units, kh = w / (d / EW), c = (w % (d / EW)) * EW;
      const T* src = row + (p.hq + p.hkv) * d + kh * d;
      T* dst = static_cast<T*>(p.v_pool) + ((p.layer_base + slot / p.bs) * p.hkv + kh) * p.bs * d + (slot % p.bs) * d;
      st<T, EW>(dst + c, ld<T, EW>(src + c));
    }
  }
}

template <typename T>
int launch(const RopeParams& p, int64_t n, bool vec16, cudaStream_t st) {
  const int threads = 128;
  if (vec16)
    rope_append_kernel<T, 8><<<(unsigned)n, threads, 0, st>>>(p);
  else
    rope_append_kernel<T, 2><<<(unsigned)n, threads, 0, st>>>(p);
  return launch_status();
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int pkv_rope_append(const pkv_pool* pool, int32_t layer, const void* qkv, int64_t qkv_stride,
                               int64_t n_tokens, int32_t num_q_heads, const int64_t* positions, const void* cos_table,
                               const void* sin_table, int64_t max_positions, void* q_out, int64_t q_out_stride_t,
                               int64_t q_out_stride_h, void* k_out, int64_t k_out_stride_t, int64_t k_out_stride_h,
                               const int64_t* slot_mapping, int32_t* status_dev, pkv_stream_t stream) {
  if (!pool || !qkv || !positions || !cos_table || !sin_table || !q_out || n_tokens < 0 || num_q_heads <= 0 ||
      max_positions <= 0)
    return PKV_ERR_INVALID_ARGUMENT;
  const int d = pool->head_dim, hkv = pool->num_kv_heads;
  if (d <= 0 || d % 4 || hkv <= 0 || num_q_heads % hkv) return PKV_ERR_INVALID_ARGUMENT;
  if (slot_mapping && (layer < 0 || layer >= pool->num_layers || !pool->k || !pool->v)) return PKV_ERR_INVALID_ARGUMENT;
  if (!slot_mapping && !k_out) return PKV_ERR_INVALID_ARGUMENT;  // the rotated keys must go somewhere
  if (pool->dtype != PKV_F16 && pool->dtype != PKV_BF16) return PKV_ERR_UNSUPPORTED;
  if (qkv_stride < (int64_t)(num_q_heads + 2 * hkv) * d) return PKV_ERR_INVALID_ARGUMENT;
  if (n_tokens == 0) return PKV_OK;
  if (n_tokens > 0x7fffffff) return PKV_ERR_INVALID_ARGUMENT;
  RopeParams p;
  p.qkv = qkv;
  p.positions = positions;
  p.cos = cos_table;
  p.sin = sin_table;
  p.q_out = q_out;
  p.k_out = k_out;
  p.k_pool = pool->k;
  p.v_pool = pool->v;
  p.slots = slot_mapping;
  p.status = status_dev;
  p.qkv_stride = qkv_stride;
  p.q_st = q_out_stride_t;
  p.q_sh = q_out_stride_h;
  p.k_st = k_out ? k_out_stride_t : 0;
  p.k_sh = k_out ? k_out_stride_h : 0;
  p.max_positions = max_positions;
  p.layer_base = slot_mapping ? (int64_t)layer * pool->num_blocks_total : 0;
  p.hq = num_q_heads;
  p.hkv = hkv;
  p.d = d;
  p.bs = pool->block_size;
  p.nbt = pool->num_blocks_total;
  // 16-byte accesses when every base and stride is a multiple of 8 elements.
  const uintptr_t addr = reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(cos_table) |
                         reinterpret_cast<uintptr_t>(sin_table) | reinterpret_cast<uintptr_t>(q_out) |
                         reinterpret_cast<uintptr_t>(k_out) | (slot_mapping ? reinterpret_cast<uintptr_t>(pool->k) |
                                                                                 reinterpret_cast<uintptr_t>(pool->v)
                                                                           : 0);
  const int64_t strides = qkv_stride | q_out_stride_t | q_out_stride_h | p.k_st | p.k_sh;
  const bool vec16 = (addr & 15) == 0 && (strides & 7) == 0 && d % 16 == 0;
  if (!vec16 && ((addr & 3) || (strides & 1))) return PKV_ERR_INVALID_ARGUMENT;  // pairs need 4-byte alignment
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return pool->dtype == PKV_F16 ? launch<__half>(p, n_tokens, vec16, st) : launch<__nv_bfloat16>(p, n_tokens, vec16, st);
}
