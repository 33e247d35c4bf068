// Greedy next-token selection fused with the LM head: token_ids[b] = argmax_v (h_b . W_v),
// the logits rounded to the model dtype first, the first index among equal maxima, so
// that the result is the reference's
//     logits = F.linear(hidden, weight).float()                  (engine/model.py:321-323,
//     tokens = logits.argmax(dim=-1)                                engine/engine.py:123)
// for an all-greedy batch (engine/sampler.py:27-31) without the [B, vocab] logits ever
// reaching memory.
//
// It is HBM-bound on the weight (vocab x hidden 16-bit values, 272 MB for Qwen2.5-0.5B's
// tied 151936 x 896 embedding), which is streamed exactly once. CTA g of the persistent
// grid owns a contiguous range of 64-row vocab units and walks it in chunks of up to 256
// rows:
//   * one copy warp streams 64-wide K stages of the chunk's weight rows and of the hidden
//     states (re-read from L2 per chunk; rows past the batch arrive as zeros) by TMA into
//     two rings, 4-5 stages of weight rows and 3 of hidden rows; with PKV_LM_WEIGHT_READY
//     the weight of the first stages is requested
//     before the wait for the previous kernel (programmatic dependent launch), the hidden
//     states always after it;
//   * one thread issues tcgen05.mma kind::f16 (A = hidden rows, M = 128 per tile; B = weight
//     rows, N = the chunk's rows; fp32 accumulators in TMEM: two 256-column chunk buffers
//     for one M tile, one 512-column buffer for two);
//   * four epilogue warps own one batch row per TMEM lane: each rounds its row's logits
//     to the model dtype and keeps the largest (first on ties), with one M tile while the
//     next chunk's MMAs run.
// The CTAs combine through a 64-bit atomic max per batch row on (ordered logit bits,
// ~index); the last CTA to take the ticket writes the token ids and leaves the workspace
// zeroed for the next call.
#include <algorithm>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "tcgen05.cuh"

namespace pkv {
namespace {

constexpr int kUnit = 64;     // vocab rows per unit (one TMA box of the weight)
constexpr int kKB = 64;       // K elements per stage: one 128-byte swizzled row
constexpr int kThreads = 192;  // copy warp, MMA warp, 4 epilogue warps
constexpr int kMaxBatch = 256;

// MT 128-row M tiles of batch rows. Chunks are 256 vocab rows; their fp32 accumulators
// (MT x 256 columns) fill the 512 TMEM columns twice over for one M tile, so the epilogue of
// one chunk overlaps the MMAs of the next, and once for two (measured: faster than two
// buffers of 128-row chunks, whose hidden rows, re-read per chunk, cost twice as much).
// The weight and the hidden rows of a K stage travel in separate rings: the weight comes
// from HBM and needs the deeper one (WS stages in flight), the hidden rows hit L2.
template <int MT>
struct LmShape {
  static constexpr int NCOLS = 512;
  static constexpr int NC = 256;                      // vocab rows per chunk (MMA N)
  static constexpr int CU = NC / kUnit;               // units per chunk
  static constexpr int BUF_COLS = MT * NC;            // TMEM columns per chunk buffer
  static constexpr int NBUF = NCOLS / BUF_COLS;       // 2 for one M tile, 1 for two
  static constexpr int A_BYTES = MT * 128 * 128;      // hidden: MT tiles of 128 rows x 64 K
  static constexpr int B_BYTES = NC * 128;            // weight: NC rows x 64 K
  static constexpr int WS = MT == 1 ? 5 : 4;          // weight stages (32 KB each)
  static constexpr int HS = 3;                        // hidden stages
  static constexpr int NBARS = 2 * WS + HS + 2 * NBUF + 1;
  static constexpr int SMEM = 1024 + WS * B_BYTES + HS * A_BYTES + NBARS * 8 + 16;
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

struct LmParams {
  int batch, vocab, hidden, n_units;
  int weight_ready;          // the weight was not written by the previous kernel in the stream
  unsigned long long* best;  // [batch] ordered key << 32 | ~index; zero between calls
  int32_t* ticket;           // zero between calls
  int64_t* ids;              // [batch]
  float* max_logits;         // [batch] or null
  int32_t* status;
};

// Order-preserving 16-bit key of a logit rounded to the model dtype (sign-magnitude bits
// mapped to unsigned order); NaN is the largest, as torch.argmax treats it.
template <typename T>
__device__ __forceinline__ uint32_t logit_key(float v) {
  uint32_t x;
  if constexpr (Dt<T>::code == PKV_BF16) {
    x = __bfloat16_as_ushort(__float2bfloat16_rn(v));
  } else {
    x = __half_as_ushort(__float2half_rn(v));
  }
  const uint32_t k = (x & 0x8000u) ? (~x & 0xFFFFu) : (x | 0x8000u);
  return v != v ? 0xFFFFu : k;
}

template <typename T>
__device__ __forceinline__ float key_value(uint32_t k) {
  const unsigned short x = (unsigned short)((k & 0x8000u) ? (k ^ 0x8000u) : (~k & 0xFFFFu));
  if constexpr (Dt<T>::code == PKV_BF16) {
    return __bfloat162float(__ushort_as_bfloat16(x));
  } else {
    return __half2float(__ushort_as_half(x));
  }
}

template <typename T, int MT>
__global__ void __launch_bounds__(kThreads, 1)
    lm_head_argmax_kernel(const __grid_constant__ CUtensorMap tmap_h, const __grid_constant__ CUtensorMap tmap_w,
                          const LmParams p) {
  using S = LmShape<MT>;
  constexpr int WS = S::WS, HS = S::HS, NBUF = S::NBUF;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring_w = smem;                          // [WS][B_BYTES]
  uint8_t* ring_h = smem + WS * S::B_BYTES;        // [HS][A_BYTES]
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring_h + HS * S::A_BYTES);
  uint64_t* w_full = bars;                // [WS] a stage's weight rows landed
  uint64_t* h_full = w_full + WS;         // [HS] a stage's hidden rows landed
  uint64_t* done = h_full + HS;           // [WS] the MMAs of stage j completed (frees both of its slots)
  uint64_t* acc_full = done + WS;         // [NBUF] a chunk's accumulators are final
  uint64_t* acc_empty = acc_full + NBUF;  // [NBUF] the epilogue warps read a chunk buffer
  uint64_t* mma_done = acc_empty + NBUF;  // every MMA of the CTA completed (before TMEM is freed)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + S::NBARS);
  int* s_last = reinterpret_cast<int*>(tslot + 1);
  auto stage_a = [&](int j) { return ring_h + (j % HS) * S::A_BYTES; };
  auto stage_b = [&](int j) { return ring_w + (j % WS) * S::B_BYTES; };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, g = blockIdx.x;
  const int per = p.n_units / G, rem = p.n_units % G;
  const int u0 = g * per + min(g, rem);          // this CTA's first unit
  const int nu = per + (g < rem ? 1 : 0);        // and how many (>= 1: the grid has <= n_units CTAs)
  const int n_chunks = (nu + S::CU - 1) / S::CU;
  const int kst = p.hidden / kKB;                // K stages per chunk
  const int total = n_chunks * kst;
  auto chunk_units = [&](int c) { return min(S::CU, nu - c * S::CU); };

  if (tid == 0) {
    for (int i = 0; i < WS; ++i) {
      mbar_init(&w_full[i], 1);
      mbar_init(&done[i], 1);
    }
    for (int i = 0; i < HS; ++i) mbar_init(&h_full[i], 1);
    for (int i = 0; i < NBUF; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, S::NCOLS);
    tc_fence_before_sync();
  }
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tslot;
  const uint64_t deadline = global_ns() + kWaitBudgetNs;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA copies
    if (lane == 0) {
      prefetch_tensormap(&tmap_h);
      prefetch_tensormap(&tmap_w);
    }
    const uint64_t stream_once = policy_evict_first(), reused = policy_evict_last();
    auto issue_w = [&](int j) {  // stage j's weight rows into slot j % WS
      const int c = j / kst, ks = j % kst, cu = chunk_units(c);
      uint64_t* bar = &w_full[j % WS];
      if (lane == 0) mbar_arrive_expect_tx(bar, cu * kUnit * 128);
      __syncwarp();
      if (lane < cu)
        tma_load_2d(stage_b(j) + lane * kUnit * 128, &tmap_w, ks * kKB, (u0 + c * S::CU + lane) * kUnit, bar,
                    stream_once);
    };
    auto issue_h = [&](int j) {  // stage j's hidden rows into slot j % HS
      const int ks = j % kst;
      uint64_t* bar = &h_full[j % HS];
      if (lane == 0) mbar_arrive_expect_tx(bar, S::A_BYTES);
      __syncwarp();
      if (lane < MT) tma_load_2d(stage_a(j) + lane * 128 * 128, &tmap_h, ks * kKB, lane * 128, bar, reused);
    };
    // The first WS weight stages (before the wait for the previous kernel when the weight is
    // known ready) and HS hidden stages; then, as the MMAs of stage c complete, the slots of
    // stage c take stage c + HS's hidden rows and stage c + WS's weight rows.
    const int pw = min(total, WS), ph = min(total, HS);
    if (p.weight_ready)
      for (int j = 0; j < pw; ++j) issue_w(j);
    grid_dep_wait();  // the hidden states are the previous kernel's output
    if (!p.weight_ready)
      for (int j = 0; j < pw; ++j) issue_w(j);
    for (int j = 0; j < ph; ++j) issue_h(j);
    bool ok = true;
    for (int c = 0; c + HS < total && ok; ++c) {
      if (lane == 0 && !mbar_wait_until(&done[c % WS], (c / WS) & 1, deadline)) ok = false;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      issue_h(c + HS);
      if (c + WS < total) issue_w(c + WS);
    }
    if (!ok && lane == 0) report(p.status, PKV_ERR_TIMEOUT);
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issue
    if (lane == 0) {
      constexpr bool kBf16 = Dt<T>::code == PKV_BF16;
      bool ok = true;
      int j = 0;
      for (int c = 0; c < n_chunks && ok; ++c) {
        const int b = c % NBUF;
        const uint32_t idesc = umma_idesc_f16(kBf16, false, 128, chunk_units(c) * kUnit);
        if (c >= NBUF && !mbar_wait_until(&acc_empty[b], ((c / NBUF) - 1) & 1, deadline)) ok = false;
        tc_fence_after_sync();
        const uint32_t d0 = tmem + (uint32_t)(b * S::BUF_COLS);
        for (int ks = 0; ks < kst && ok; ++ks, ++j) {
          if (!mbar_wait_until(&w_full[j % WS], (j / WS) & 1, deadline) ||
              !mbar_wait_until(&h_full[j % HS], (j / HS) & 1, deadline)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
#pragma unroll
          for (int kk = 0; kk < kKB / 16; ++kk) {
            const uint64_t bd = umma_desc_sw128(smem_u32(stage_b(j) + kk * 32), 16, 1024);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
              const uint64_t ad = umma_desc_sw128(smem_u32(stage_a(j) + mt * 128 * 128 + kk * 32), 16, 1024);
              umma_f16_ss(d0 + mt * S::NC, ad, bd, idesc, ks > 0 || kk > 0);
            }
          }
          umma_commit(&done[j % WS]);
        }
        if (ok) umma_commit(&acc_full[b]);
      }
      if (!ok) report(p.status, PKV_ERR_TIMEOUT);
      if (total > 0) umma_commit(mma_done); else mbar_arrive(mma_done);
    }
  } else {
    // ---------------------------------------------------------------- epilogue warps
    const int q = warp % 4;                     // TMEM lane quarter of this warp
    const int r = q * 32 + lane;                // batch row within an M tile
    const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16);
    uint32_t bk[MT];
    int bi[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) bk[mt] = 0, bi[mt] = -1;
    bool ok = true;
    for (int c = 0; c < n_chunks; ++c) {
      const int b = c % NBUF, cu = chunk_units(c);
      if (ok && !mbar_wait_until(&acc_full[b], (c / NBUF) & 1, deadline)) ok = false;
      tc_fence_after_sync();
      const int v0 = (u0 + c * S::CU) * kUnit;  // vocab index of the chunk's first row
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        for (int cc = 0; cc < cu * (kUnit / 32); ++cc) {
          uint32_t v[32];
          tmem_ld32(tl + (uint32_t)(b * S::BUF_COLS + mt * S::NC + cc * 32), v);
          tmem_wait_ld();
          const int i0 = v0 + cc * 32;
          if (i0 + 32 <= p.vocab) {
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const uint32_t k = logit_key<T>(__uint_as_float(v[e]));
              if (k > bk[mt]) bk[mt] = k, bi[mt] = i0 + e;
            }
          } else {  // the last unit's rows past the vocabulary are zero-filled: skip them
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const uint32_t k = logit_key<T>(__uint_as_float(v[e]));
              if (i0 + e < p.vocab && k > bk[mt]) bk[mt] = k, bi[mt] = i0 + e;
            }
          }
        }
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
    if (!ok) report(p.status, PKV_ERR_TIMEOUT);
    grid_dep_wait();  // the workspace and the outputs may still be read by the previous kernel
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int row = mt * 128 + r;
      if (row < p.batch && bi[mt] >= 0)
        atomicMax(&p.best[row], ((unsigned long long)bk[mt] << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)bi[mt]));
    }
    fence_acq_rel_gpu();  // this thread's maxima before the ticket below
    named_barrier_sync(1, 128);
    if (warp == 2 && lane == 0) *s_last = atom_add_acq_rel_gpu(p.ticket, 1) == G - 1;
    named_barrier_sync(1, 128);
    if (*s_last) {  // every other CTA's maxima are in: publish and leave the workspace zeroed
      fence_acq_rel_gpu();
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int row = mt * 128 + r;
        if (row < p.batch) {
          const unsigned long long v = atomicExch(&p.best[row], 0ull);
          if (v == 0ull) report(p.status, PKV_ERR_TIMEOUT);  // a CTA gave up before its maxima
          p.ids[row] = (int64_t)(0xFFFFFFFFu - (uint32_t)(v & 0xFFFFFFFFull));
          if (p.max_logits) p.max_logits[row] = key_value<T>((uint32_t)(v >> 32));
        }
      }
      if (warp == 2 && lane == 0) st_relaxed_gpu(p.ticket, 0);
    }
  }
  __syncthreads();
  if (warp == 1) {
    if (!mbar_wait_until(mma_done, 0, global_ns() + kWaitBudgetNs) && lane == 0) report(p.status, PKV_ERR_TIMEOUT);
    tc_fence_after_sync();
    tmem_dealloc(tmem, S::NCOLS);
  }
}

// Tensor maps are encoded on the host (a few microseconds); the weight's is reused across
// calls, the hidden states' whenever the same buffer comes back (as in a CUDA graph).
struct MatrixMapKey {
  const void* base;
  int dtype;
  uint64_t inner, rows, stride;
  uint32_t box_rows;
  bool operator==(const MatrixMapKey& o) const { return std::memcmp(this, &o, sizeof(*this)) == 0; }
};
std::mutex g_lm_mutex;
std::vector<std::pair<MatrixMapKey, CUtensorMap>> g_lm_maps;

int matrix_map(CUtensorMap* out, const void* base, int dtype, uint64_t inner, uint64_t rows, uint64_t stride_bytes,
               uint32_t box_rows) {
  MatrixMapKey k;
  std::memset(&k, 0, sizeof(k));
  k.base = base, k.dtype = dtype, k.inner = inner, k.rows = rows, k.stride = stride_bytes, k.box_rows = box_rows;
  std::lock_guard<std::mutex> lock(g_lm_mutex);
  for (const auto& e : g_lm_maps) {
    if (e.first == k) {
      *out = e.second;
      return PKV_OK;
    }
  }
  CUtensorMap m;
  const int rc = make_matrix_tensor_map(&m, base, dtype, inner, rows, stride_bytes, kKB, box_rows);
  if (rc != PKV_OK) return rc;
  if (g_lm_maps.size() >= 32) g_lm_maps.erase(g_lm_maps.begin());
  g_lm_maps.emplace_back(k, m);
  *out = m;
  return PKV_OK;
}

template <typename T, int MT>
int launch_lm_head(const CUtensorMap& th, const CUtensorMap& tw, const LmParams& p, cudaStream_t stream) {
  using S = LmShape<MT>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e =
        cudaFuncSetAttribute(lm_head_argmax_kernel<T, MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM);
    if (e != cudaSuccess) return cuda_status(e);
    configured = true;
  }
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3((unsigned)std::min(p.n_units, num_sms()));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = S::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, lm_head_argmax_kernel<T, MT>, th, tw, p));
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int64_t pkv_lm_head_argmax_workspace_bytes(int32_t batch) {
  return batch < 0 ? 0 : 8 + 8 * (int64_t)batch;
}

extern "C" int pkv_lm_head_argmax(const void* hidden, int64_t hidden_stride, int32_t batch, const void* weight,
                                  int64_t weight_stride, int32_t vocab, int32_t hidden_size, int32_t dtype,
                                  int64_t* token_ids, float* max_logits, void* workspace, int64_t workspace_bytes,
                                  int32_t flags, int32_t* status_dev, pkv_stream_t stream) {
  if (!hidden || !weight || !token_ids || !workspace) return PKV_ERR_INVALID_ARGUMENT;
  if (batch < 0 || vocab <= 0 || hidden_size <= 0) return PKV_ERR_INVALID_ARGUMENT;
  if (dtype != PKV_F16 && dtype != PKV_BF16) return PKV_ERR_UNSUPPORTED;
  if (batch > kMaxBatch || hidden_size % kKB != 0) return PKV_ERR_UNSUPPORTED;
  if (hidden_stride < hidden_size || weight_stride < hidden_size || hidden_stride % 8 || weight_stride % 8)
    return PKV_ERR_INVALID_ARGUMENT;
  auto aligned = [](const void* ptr, uintptr_t a) { return (reinterpret_cast<uintptr_t>(ptr) & (a - 1)) == 0; };
  if (!aligned(hidden, 16) || !aligned(weight, 16) || !aligned(token_ids, 8) || !aligned(workspace, 8) ||
      (max_logits && !aligned(max_logits, 4)))
    return PKV_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < pkv_lm_head_argmax_workspace_bytes(batch)) return PKV_ERR_WORKSPACE;
  if (batch == 0) return PKV_OK;
  const int mt = batch <= 128 ? 1 : 2;
  CUtensorMap th, tw;
  int rc = matrix_map(&th, hidden, dtype, (uint64_t)hidden_size, (uint64_t)batch, (uint64_t)hidden_stride * 2, 128);
  if (rc == PKV_OK)
    rc = matrix_map(&tw, weight, dtype, (uint64_t)hidden_size, (uint64_t)vocab, (uint64_t)weight_stride * 2, kUnit);
  if (rc != PKV_OK) return rc;
  LmParams p;
  p.batch = batch, p.vocab = vocab, p.hidden = hidden_size, p.n_units = (vocab + kUnit - 1) / kUnit;
  p.weight_ready = (flags & PKV_LM_WEIGHT_READY) ? 1 : 0;
  p.ticket = reinterpret_cast<int32_t*>(workspace);
  p.best = reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(workspace) + 8);
  p.ids = token_ids, p.max_logits = max_logits, p.status = status_dev;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == PKV_F16)
    return mt == 1 ? launch_lm_head<__half, 1>(th, tw, p, st) : launch_lm_head<__half, 2>(th, tw, p, st);
  return mt == 1 ? launch_lm_head<__nv_bfloat16, 1>(th, tw, p, st) : launch_lm_head<__nv_bfloat16, 2>(th, tw, p, st);
}
