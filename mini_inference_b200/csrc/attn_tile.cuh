// One 16-key step of flash attention for one warp, shared by the decode and the
// prefill kernels: S = Q K^T on a staged K tile, mask, online softmax update, and
// O += P V on the staged V tile, all on mma.sync m16n8k16 with fp32 accumulation.
//
// Tiles come from the 5-D TMA copy of one (layer, block, head) of the pool with a
// 128-byte swizzle (see make_pool_tensor_map). Element (token t, dim d) of a
// 16 x D tile lives in 128-byte row (d / 64) * 16 + t, column d % 64.
//
// Fragment ownership follows the PTX m16n8k16 layouts: lane = 4 * g + t4 holds
// rows g and g + 8 of the 16-row tile, and key columns 2 * t4, 2 * t4 + 1 of each
// 8-key n-tile. The running row max m_r, row sum l_r (lane-partial: reduce over
// the quad at the end) and output accumulators o are per lane.
#pragma once

#include "common.cuh"

namespace pkv {

template <int D>
__device__ inline uint32_t tile_addr(uint32_t base, int key, int unit) {
  const uint32_t r = (unit >> 3) * 16 + key;
  return base + swz128(r, (unit & 7) * 8);
}

// allowed(row, key) -> bool, row in [0, 16), key = absolute key position.
template <typename T, int D, typename Mask>
__device__ inline void attend_tile16(const uint32_t (&qa)[D / 16][4], uint32_t kbase, uint32_t vbase, int key0,
                                     const Mask& allowed, float scale_log2, float (&m_r)[2], float (&l_r)[2],
                                     float (&o)[D / 8][4]) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  float s[2][4];
#pragma unroll
  for (int n = 0; n < 2; ++n) {
    s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int k2 = 0; k2 < D / 32; ++k2) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4(tile_addr<D>(kbase, 8 * n + (lane & 7), 4 * k2 + (lane >> 3)), b0, b1, b2, b3);
      mma16816<T>(s[n], qa[2 * k2], b0, b1);
      mma16816<T>(s[n], qa[2 * k2 + 1], b2, b3);
    }
  }
#pragma unroll
  for (int n = 0; n < 2; ++n) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int key = key0 + 8 * n + 2 * t4 + (e & 1);
      const int row = g + 8 * (e >> 1);
      s[n][e] = allowed(row, key) ? s[n][e] * scale_log2 : -INFINITY;
    }
  }
  float mx[2] = {fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1])),
                 fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]))};
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
    mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
  }
  float alpha[2], mref[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float mn = fmaxf(m_r[i], mx[i]);
    // A row with no allowed key so far keeps m = -inf; use 0 as the reference so that
    // exp2(-inf - 0) = 0 instead of exp2(-inf + inf) = NaN.
    mref[i] = mn == -INFINITY ? 0.f : mn;
    alpha[i] = ex2(m_r[i] - mref[i]);
    m_r[i] = mn;
  }
  float ps[2] = {0.f, 0.f};
#pragma unroll
  for (int n = 0; n < 2; ++n) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      s[n][e] = ex2(s[n][e] - mref[e >> 1]);
      ps[e >> 1] += s[n][e];
    }
  }
  l_r[0] = l_r[0] * alpha[0] + ps[0];
  l_r[1] = l_r[1] * alpha[1] + ps[1];
#pragma unroll
  for (int j = 0; j < D / 8; ++j) {
    o[j][0] *= alpha[0];
    o[j][1] *= alpha[0];
    o[j][2] *= alpha[1];
    o[j][3] *= alpha[1];
  }
  // P enters the tensor cores in the storage type. fp16 keeps 11 significant bits of
  // each weight; bf16 only 8, which alone moves short-context outputs by several bf16
  // steps, so for bf16 P is split as hi + lo (both bf16, ~16 bits together) and V is
  // multiplied by both. Decode is memory-bound, so the second pass is free there.
  constexpr bool kSplitP = !Dt<T>::kExactP;
  uint32_t pa[4], pl[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int n = i >> 1, e = (i & 1) * 2;
    pa[i] = Dt<T>::pack(s[n][e], s[n][e + 1]);
    if (kSplitP) {
      const float2 hi = Dt<T>::unpack(pa[i]);
      pl[i] = Dt<T>::pack(s[n][e] - hi.x, s[n][e + 1] - hi.y);
    }
  }
#pragma unroll
  for (int jj = 0; jj < D / 16; ++jj) {
    uint32_t b0, b1, b2, b3;
    ldsm_x4_t(tile_addr<D>(vbase, (lane & 7) + 8 * ((lane >> 3) & 1), 2 * jj + (lane >> 4)), b0, b1, b2, b3);
    mma16816<T>(o[2 * jj], pa, b0, b1);
    mma16816<T>(o[2 * jj + 1], pa, b2, b3);
    if (kSplitP) {
      mma16816<T>(o[2 * jj], pl, b0, b1);
      mma16816<T>(o[2 * jj + 1], pl, b2, b3);
    }
  }
}

// Row sums are lane-partial during the loop; complete them across the quad.
__device__ inline void finish_row_sums(float (&l_r)[2]) {
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    l_r[i] += __shfl_xor_sync(0xffffffffu, l_r[i], 1);
    l_r[i] += __shfl_xor_sync(0xffffffffu, l_r[i], 2);
  }
}

}  // namespace pkv
