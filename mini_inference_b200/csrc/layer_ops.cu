// The decoder layer's elementwise glue around the paged-KV path, one launch per step of it.
//
// The reference's Qwen2 decoder layer (engine/model.py:266-280) runs, per layer and
// forward, two RMSNorms of eight eager launches each (float, pow, mean, add, rsqrt, mul,
// cast, weight mul: engine/model.py:162-166), two residual adds and the MLP's SiLU and
// multiply (engine/model.py:262-264). At serving batch sizes each of those launches
// moves a few hundred KB and costs its launch and ramp; together they take about half of
// a 0.5B-shaped decode step's GPU time. Here:
//   pkv_add_rms_norm: h = r(x + residual) (optional, written back to the residual
//     stream), then out = r(w * r(h * rsqrt(mean(h^2) + eps))), statistics in float32;
//   pkv_silu_mul: out = r(r(silu(g)) * u) for gate_up = [g | u], silu(g) = g / (1 + e^-g)
//     in float32,
// where r() rounds to the model dtype, at the points where the reference's eager ops
// round. The residual add and every rounding match the reference's bit for bit; the sum
// of squares runs in a different order than torch's mean reduction (float32 either way).
//
// Rows are independent and short (hidden 896 .. 8192 elements): one CTA per row, each
// thread holding P 16-byte packs of the row in registers between the statistic and the
// scaling, the sum reduced by warp shuffles and one shared-memory step. The SiLU kernel
// is a flat grid-stride loop over 16-byte packs of the gate half and the up half.
#include "common.cuh"

namespace pkv {
namespace {

template <typename T, int EW> struct alignas(EW * sizeof(T)) Vec {
  T v[EW];
};

struct NormParams {
  const void* x;            // [rows, hidden] of T, or with splits > 0: float partials [splits][rows][hidden]
  int64_t split_stride;     // elements between the partials of consecutive splits
  int32_t splits;
  const void* residual_in;
  void* residual_out;
  const void* weight;
  void* out;
  int64_t x_stride, rin_stride, rout_stride, out_stride;
  int32_t hidden;
  float eps;
};

// PART: x arrives as split-K partial sums in float32 (a GEMM cut along K); their sum,
// slice by slice in order and rounded to T, is the projection's output the reference's
// F.linear would have rounded.
template <typename T, int EW, int P, bool PART>
__global__ void __launch_bounds__(1024) add_rms_norm_kernel(const NormParams p) {
  __shared__ float s_part[32];
  grid_dep_launch_dependents();  // a kernel that reads only weights may start early
  const int64_t row = blockIdx.x;
  const int packs = p.hidden / EW;
  const T* x = PART ? nullptr : static_cast<const T*>(p.x) + row * p.x_stride;
  const T* rin = p.residual_in ? static_cast<const T*>(p.residual_in) + row * p.rin_stride : nullptr;
  T* rout = p.residual_out ? static_cast<T*>(p.residual_out) + row * p.rout_stride : nullptr;
  float h[P][EW];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < P; ++k) {
    const int c = threadIdx.x + k * blockDim.x;
    if (c < packs) {
      Vec<T, EW> a;
      if constexpr (PART) {
        const float* xp = static_cast<const float*>(p.x) + row * p.x_stride + (int64_t)c * EW;
        float acc[EW];
#pragma unroll
        for (int e = 0; e < EW; ++e) acc[e] = 0.f;
        for (int sp = 0; sp < p.splits; ++sp) {
          const float* q = xp + sp * p.split_stride;
#pragma unroll
          for (int e = 0; e < EW; e += (EW >= 4 ? 4 : 1)) {
            if constexpr (EW >= 4) {
              const float4 v = *reinterpret_cast<const float4*>(q + e);
              acc[e] += v.x, acc[e + 1] += v.y, acc[e + 2] += v.z, acc[e + 3] += v.w;
            } else {
              acc[e] += q[e];
            }
          }
        }
#pragma unroll
        for (int e = 0; e < EW; ++e) a.v[e] = Dt<T>::from_f(acc[e]);
      } else {
        a = reinterpret_cast<const Vec<T, EW>*>(x)[c];
      }
      if (rin) {
        const Vec<T, EW> b = reinterpret_cast<const Vec<T, EW>*>(rin)[c];
#pragma unroll
        for (int e = 0; e < EW; ++e) a.v[e] = Dt<T>::from_f(Dt<T>::to_f(a.v[e]) + Dt<T>::to_f(b.v[e]));
      }
      if (rout) reinterpret_cast<Vec<T, EW>*>(rout)[c] = a;
#pragma unroll
      for (int e = 0; e < EW; ++e) {
        h[k][e] = Dt<T>::to_f(a.v[e]);
        ss = __fadd_rn(ss, __fmul_rn(h[k][e], h[k][e]));  // pow(2) rounded, then summed
      }
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = (blockDim.x + 31) >> 5;
  if (lane == 0) s_part[warp] = ss;
  __syncthreads();
  float tot = lane < nwarps ? s_part[lane] : 0.f;
#pragma unroll
  for (int o = 16; o; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
  const float rs = rsqrtf(tot / (float)p.hidden + p.eps);
  const Vec<T, EW>* w = static_cast<const Vec<T, EW>*>(p.weight);
  Vec<T, EW>* out = reinterpret_cast<Vec<T, EW>*>(static_cast<T*>(p.out) + row * p.out_stride);
#pragma unroll
  for (int k = 0; k < P; ++k) {
    const int c = threadIdx.x + k * blockDim.x;
    if (c < packs) {
      const Vec<T, EW> wk = w[c];
      Vec<T, EW> y;
#pragma unroll
      for (int e = 0; e < EW; ++e) {
        const T n = Dt<T>::from_f(h[k][e] * rs);
        y.v[e] = Dt<T>::from_f(Dt<T>::to_f(wk.v[e]) * Dt<T>::to_f(n));
      }
      out[c] = y;
    }
  }
}

template <typename T, int EW, bool PART>
int launch_norm(const NormParams& p, int64_t rows, cudaStream_t st) {
  const int packs = p.hidden / EW;
  // Fewest packs per thread that keep the CTA at or below 1024 threads.
  int P = 1;
  while (P < 8 && (packs + P - 1) / P > 1024) P *= 2;
  if ((packs + P - 1) / P > 1024) return PKV_ERR_UNSUPPORTED;
  const int threads = (((packs + P - 1) / P) + 31) / 32 * 32;
  const unsigned grid = (unsigned)rows;
  switch (P) {
    case 1: add_rms_norm_kernel<T, EW, 1, PART><<<grid, threads, 0, st>>>(p); break;
    case 2: add_rms_norm_kernel<T, EW, 2, PART><<<grid, threads, 0, st>>>(p); break;
    case 4: add_rms_norm_kernel<T, EW, 4, PART><<<grid, threads, 0, st>>>(p); break;
    default: add_rms_norm_kernel<T, EW, 8, PART><<<grid, threads, 0, st>>>(p); break;
  }
  return launch_status();
}

struct SiluParams {
  const void* gate_up;
  void* out;
  int64_t gu_stride, out_stride, rows;
  int32_t inter;
};

template <typename T, int EW>
__global__ void __launch_bounds__(256) silu_mul_kernel(const SiluParams p) {
  const int per_row = p.inter / EW;
  const int64_t total = p.rows * per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / per_row;
    const int c = (int)(i - row * per_row);
    const T* g = static_cast<const T*>(p.gate_up) + row * p.gu_stride;
    const Vec<T, EW> gv = reinterpret_cast<const Vec<T, EW>*>(g)[c];
    const Vec<T, EW> uv = reinterpret_cast<const Vec<T, EW>*>(g + p.inter)[c];
    Vec<T, EW> y;
#pragma unroll
    for (int e = 0; e < EW; ++e) {
      const float x = Dt<T>::to_f(gv.v[e]);
      const T s = Dt<T>::from_f(x / (1.0f + expf(-x)));
      y.v[e] = Dt<T>::from_f(Dt<T>::to_f(s) * Dt<T>::to_f(uv.v[e]));
    }
    reinterpret_cast<Vec<T, EW>*>(static_cast<T*>(p.out) + row * p.out_stride)[c] = y;
  }
}

template <typename T, int EW>
int launch_silu(const SiluParams& p, cudaStream_t st) {
  const int threads = 256;
  const int64_t work = p.rows * (p.inter / EW);
  static int sms_of[64];  // SM count per device, looked up once
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < 64) {
    if (!sms_of[dev]) cudaDeviceGetAttribute(&sms_of[dev], cudaDevAttrMultiProcessorCount, dev);
    if (sms_of[dev] > 0) sms = sms_of[dev];
  }
  // Enough CTAs for one pack per thread up to 8 resident CTAs per SM; a grid-stride loop beyond.
  const int64_t want = (work + threads - 1) / threads;
  const unsigned grid = (unsigned)(want < (int64_t)sms * 8 ? want : (int64_t)sms * 8);
  silu_mul_kernel<T, EW><<<grid, threads, 0, st>>>(p);
  return launch_status();
}

bool aligned(const void* ptr, int bytes) { return (reinterpret_cast<uintptr_t>(ptr) % bytes) == 0; }

}  // namespace
}  // namespace pkv

using namespace pkv;

namespace pkv {
namespace {

// splits == 0: x is [rows, hidden] of the model dtype; else float32 partials [splits][rows][hidden].
int norm_entry(int32_t dtype, const void* x, int64_t x_stride, int32_t splits, int64_t split_stride,
               const void* residual_in, int64_t residual_in_stride, void* residual_out, int64_t residual_out_stride,
               const void* weight, void* out, int64_t out_stride, int64_t rows, int32_t hidden, float eps,
               pkv_stream_t stream) {
  if (!x || !weight || !out || rows < 0 || hidden <= 0 || !(eps >= 0.f) || splits < 0) return PKV_ERR_INVALID_ARGUMENT;
  if (dtype != PKV_F16 && dtype != PKV_BF16) return PKV_ERR_UNSUPPORTED;
  if (x_stride < hidden || out_stride < hidden || (residual_in && residual_in_stride < hidden) ||
      (residual_out && residual_out_stride < hidden))
    return PKV_ERR_INVALID_ARGUMENT;
  if (splits > 0 && split_stride < rows * x_stride) return PKV_ERR_INVALID_ARGUMENT;
  if (rows == 0) return PKV_OK;
  if (rows > 0x7fffffff) return PKV_ERR_INVALID_ARGUMENT;
  NormParams p;
  p.x = x;
  p.split_stride = split_stride;
  p.splits = splits;
  p.residual_in = residual_in;
  p.residual_out = residual_out;
  p.weight = weight;
  p.out = out;
  p.x_stride = x_stride;
  p.rin_stride = residual_in ? residual_in_stride : 0;
  p.rout_stride = residual_out ? residual_out_stride : 0;
  p.out_stride = out_stride;
  p.hidden = hidden;
  p.eps = eps;
  // 16-byte packs when every row start is 16-byte aligned, else one element per pack.
  const int64_t strides = x_stride | out_stride | p.rin_stride | p.rout_stride | (splits ? split_stride : 0);
  const bool vec = hidden % 8 == 0 && strides % 8 == 0 && aligned(x, 16) && aligned(weight, 16) && aligned(out, 16) &&
                   (!residual_in || aligned(residual_in, 16)) && (!residual_out || aligned(residual_out, 16));
  if (!vec && (!aligned(x, splits ? 4 : 2) || !aligned(weight, 2) || !aligned(out, 2))) return PKV_ERR_INVALID_ARGUMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (splits > 0) {
    if (dtype == PKV_F16)
      return vec ? launch_norm<__half, 8, true>(p, rows, st) : launch_norm<__half, 1, true>(p, rows, st);
    return vec ? launch_norm<__nv_bfloat16, 8, true>(p, rows, st) : launch_norm<__nv_bfloat16, 1, true>(p, rows, st);
  }
  if (dtype == PKV_F16)
    return vec ? launch_norm<__half, 8, false>(p, rows, st) : launch_norm<__half, 1, false>(p, rows, st);
  return vec ? launch_norm<__nv_bfloat16, 8, false>(p, rows, st) : launch_norm<__nv_bfloat16, 1, false>(p, rows, st);
}

}  // namespace
}  // namespace pkv

extern "C" int pkv_add_rms_norm(int32_t dtype, const void* x, int64_t x_stride, const void* residual_in,
                                int64_t residual_in_stride, void* residual_out, int64_t residual_out_stride,
                                const void* weight, void* out, int64_t out_stride, int64_t rows, int32_t hidden,
                                float eps, pkv_stream_t stream) {
  return norm_entry(dtype, x, x_stride, 0, 0, residual_in, residual_in_stride, residual_out, residual_out_stride,
                    weight, out, out_stride, rows, hidden, eps, stream);
}

extern "C" int pkv_add_rms_norm_partials(int32_t dtype, const float* partials, int64_t row_stride, int32_t splits,
                                         int64_t split_stride, const void* residual_in, int64_t residual_in_stride,
                                         void* residual_out, int64_t residual_out_stride, const void* weight,
                                         void* out, int64_t out_stride, int64_t rows, int32_t hidden, float eps,
                                         pkv_stream_t stream) {
  if (splits <= 0) return PKV_ERR_INVALID_ARGUMENT;
  return norm_entry(dtype, partials, row_stride, splits, split_stride, residual_in, residual_in_stride, residual_out,
                    residual_out_stride, weight, out, out_stride, rows, hidden, eps, stream);
}

extern "C" int pkv_silu_mul(int32_t dtype, const void* gate_up, int64_t gate_up_stride, void* out, int64_t out_stride,
                            int64_t rows, int32_t intermediate, pkv_stream_t stream) {
  if (!gate_up || !out || rows < 0 || intermediate <= 0) return PKV_ERR_INVALID_ARGUMENT;
  if (dtype != PKV_F16 && dtype != PKV_BF16) return PKV_ERR_UNSUPPORTED;
  if (gate_up_stride < 2 * (int64_t)intermediate || out_stride < intermediate) return PKV_ERR_INVALID_ARGUMENT;
  if (rows == 0) return PKV_OK;
  SiluParams p;
  p.gate_up = gate_up;
  p.out = out;
  p.gu_stride = gate_up_stride;
  p.out_stride = out_stride;
  p.rows = rows;
  p.inter = intermediate;
  const bool vec = intermediate % 8 == 0 && (gate_up_stride | out_stride) % 8 == 0 && aligned(gate_up, 16) &&
                   aligned(out, 16);
  if (!vec && (!aligned(gate_up, 2) || !aligned(out, 2))) return PKV_ERR_INVALID_ARGUMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == PKV_F16) return vec ? launch_silu<__half, 8>(p, st) : launch_silu<__half, 1>(p, st);
  return vec ? launch_silu<__nv_bfloat16, 8>(p, st) : launch_silu<__nv_bfloat16, 1>(p, st);
}
