// Shared device helpers for the sm_100a paged-KV kernels: dtype traits, inline
// PTX wrappers (mbarrier, bulk tensor copies, ldmatrix, mma.sync, ex2), the
// device status word, and host-side error plumbing.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/pkv.h"

namespace pkv {

// ---------------------------------------------------------------- host-side error plumbing
void set_last_cuda_error(cudaError_t e);
int cuda_status(cudaError_t e);  // PKV_OK or PKV_ERR_CUDA (and records the message)

inline int launch_status() { return cuda_status(cudaGetLastError()); }

// ---------------------------------------------------------------- dtype traits
template <typename T> struct Dt;
template <> struct Dt<__half> {
  static constexpr int code = PKV_F16;
  static constexpr bool kExactP = true;  // softmax weights in [0, 1] keep 11 bits in fp16
  __device__ static inline uint32_t pack(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ static inline float2 unpack(uint32_t u) {
    return __half22float2(*reinterpret_cast<const __half2*>(&u));
  }
  __device__ static inline float to_f(__half x) { return __half2float(x); }
  __device__ static inline __half from_f(float x) { return __float2half_rn(x); }
};
template <> struct Dt<__nv_bfloat16> {
  static constexpr int code = PKV_BF16;
  static constexpr bool kExactP = false;  // 8 bits: the tile step splits P into hi + lo
  __device__ static inline uint32_t pack(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ static inline float2 unpack(uint32_t u) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
  }
  __device__ static inline float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ static inline __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

// ---------------------------------------------------------------- device status word
// The first error wins; later ones are dropped. Kernels never trap: a bad index is
// recorded here, the access is skipped or clamped, and the host raises.
__device__ inline void report(int32_t* status, int32_t code) {
  if (status) atomicCAS(status, 0, code);
}

// ---------------------------------------------------------------- PTX wrappers
__device__ inline uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ inline void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ inline void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ inline void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

// Named barrier `id` (1..15; 0 is __syncthreads) over `threads` threads (a multiple of 32).
__device__ inline void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// One arrival (no transaction bytes).
__device__ inline void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}

__device__ inline bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Paired fp32 arithmetic (sm_100): one instruction for two lanes of values, rounded as
// the scalar forms are.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

__device__ inline uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Every wait in a CTA shares one deadline, so a CTA waits at most this long in total.
constexpr uint64_t kWaitBudgetNs = 2000ull * 1000 * 1000;  // 2 s

// Bounded wait: polls until the phase completes or the global timer passes `deadline`,
// then returns false; the caller records PKV_ERR_TIMEOUT and stops waiting.
__device__ inline bool mbar_wait_until(uint64_t* bar, uint32_t parity, uint64_t deadline) {
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() > deadline) return false;
  }
  return true;
}

// 5-D bulk tensor copy global -> shared (no multicast), completion on an mbarrier.
__device__ inline void tma_load_5d(void* smem_dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                   int c4, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7], %8;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(smem_u32(bar)),
      "l"(policy)
      : "memory");
}

// Same copy with the default L2 policy.
__device__ inline void tma_load_5d(void* smem_dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                   int c4, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(smem_u32(bar))
      : "memory");
}

// 2-D bulk tensor copy global -> shared (no multicast) with an L2 cache policy; c0 is the
// innermost coordinate (elements), c1 the row.
__device__ inline void tma_load_2d(void* smem_dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar,
                                   uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Bulk (non-tensor) copy of `bytes` (a multiple of 16, both addresses 16-byte aligned)
// global -> shared, completing on an mbarrier (no multicast).
__device__ inline void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(smem_dst)), "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// Orders this thread's generic-proxy accesses of global memory before later async-proxy ones.
__device__ inline void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// 16-byte asynchronous global -> shared copy through L2 only (no registers held), and the
// wait for all of this thread's outstanding copies.
__device__ inline void cp_async_16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ inline void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Acquire-release fence at GPU scope (cheaper than the sequentially consistent __threadfence).
__device__ inline void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
// Atomic add with acquire and release semantics at GPU scope: earlier writes (of this
// thread, and of threads that synchronized with it first) are visible to whoever reads
// the counter afterwards, and later reads see what earlier releasers published.
__device__ inline int atom_add_acq_rel_gpu(int32_t* ptr, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(ptr), "r"(v) : "memory");
  return old;
}
__device__ inline int ld_acquire_gpu(const int32_t* ptr) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}
__device__ inline void st_relaxed_gpu(int32_t* ptr, int v) {
  asm volatile("st.relaxed.gpu.global.b32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}

__device__ inline void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ inline uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ inline uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Programmatic dependent launch (sm_90+): let the next grid in the stream start its
// CTAs now / wait until the previous grid has completed and its writes are visible.
// Both are no-ops for a launch without the programmatic-serialization attribute.
__device__ inline void grid_dep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ inline void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ inline void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ inline void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ inline void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename T>
__device__ inline void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);

template <>
__device__ inline void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <>
__device__ inline void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 2^x with the hardware's approximate exponential unit (PTX ex2.approx.ftz.f32).
__device__ inline float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Byte offset of element `col` (16-bit elements) of row `row` inside a tile whose
// rows are 128 bytes, stored with the TMA 128-byte swizzle: 16-byte unit u of row r
// lands at unit u ^ (r % 8). Tiles are 1024-byte aligned.
__device__ inline uint32_t swz128(uint32_t row, uint32_t col) {
  const uint32_t unit = (col >> 3) ^ (row & 7);
  return row * 128 + unit * 16 + (col & 7) * 2;
}

// ---------------------------------------------------------------- host: tensor maps
// 5-D tensor map over a [L, NBt, Hkv, bs, D] pool, viewed as {64, bs, D/64, Hkv, L*NBt}
// (innermost first) with a box of {64, bs, D/64, 1, 1}: one (layer, block, head) tile per
// copy, 128-byte swizzle. In shared memory the tile is [D/64][bs][64]: element (token t,
// dim d) sits in 128-byte row (d / 64) * bs + t at column d % 64, so the 8 consecutive keys
// an ldmatrix reads are 8 distinct swizzle rows (no bank conflicts for D = 64 or 128).
// heads_per_box > 1 widens the box over that many consecutive KV heads of the block:
// shared-memory layout [heads][D/64][bs][64], head h's tile at h * bs * D * 2 bytes.
// Box: 64 elements x block_size tokens x chunks_per_box 64-wide head_dim chunks (0 = all)
// x heads_per_box KV heads of one (layer, block).
int make_pool_tensor_map(CUtensorMap* map, const void* base, const pkv_pool& pool, int heads_per_box,
                         int chunks_per_box = 0);
// Cached K and V maps of a pool (one encode per pool and box shape).
bool get_pool_maps(const pkv_pool& pool, CUtensorMap* tk, CUtensorMap* tv, int heads_per_box = 1,
                   int chunks_per_box = 0);
// 2-D tensor map over a row-major [rows, inner] matrix of 16-bit elements (row stride in
// bytes, a multiple of 16) with a box of box_rows x box_inner (box_inner * 2 = 128 bytes
// for the 128-byte swizzle). Rows past `rows` read as zeros.
int make_matrix_tensor_map(CUtensorMap* map, const void* base, int dtype, uint64_t inner, uint64_t rows,
                           uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows);
// Streaming multiprocessors of the current device (queried once).
int num_sms();

}  // namespace pkv
