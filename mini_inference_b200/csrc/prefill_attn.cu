// Packed (varlen) prefill attention over the paged KV cache, prefix-cache hits included.
//
// Replaces PackedPrefillContext.attend (engine/kv_cache.py:283-297) after its
// append: the reference either runs SDPA on the packed new tokens with a
// block-diagonal causal mask, or -- with a prefix hit -- gathers every
// sequence's keys 0..end back from the cache and runs SDPA with a dense
// [N, sum of ends] mask; in both, GQA repeats each KV head 7 times
// (engine/model.py:119-123). Here every sequence's keys are read in place from
// its blocks (the new tokens were appended first, so one path serves both
// cases), and only the causal part of each sequence is visited.
//
// The contraction runs on the fifth-generation tensor cores (tcgen05) with the
// accumulators in tensor memory. One CTA takes one KV head of one sequence and TQ of
// its new tokens; the M = 128 rows of the MMA tile are those tokens x the GQA group's
// query heads (16 x 7 = 112 rows for Qwen2's group of 7), so every K/V block read
// serves the whole group. Keys stream in stages of NK = 64 (four blocks) through a
// two-stage TMA ring: S = Q K^T (M 128 x N 64, fp32 in TMEM), an online softmax by
// four warps that each own 32 TMEM lanes (one row per thread, no shuffles), P written
// to shared memory as fp16/bf16, then O_stage = P V (M 128 x N head_dim, in TMEM),
// which the softmax warps fold into their fp32 row accumulators with the running
// rescale. One warp issues the TMA copies, one thread the MMAs; mbarriers (MMA
// completion through tcgen05.commit) order the three roles. Only the causal part of
// each sequence is visited; keys past a tile's last position are masked to -inf.
#include "common.cuh"
#include "tcgen05.cuh"

namespace pkv {
namespace {

constexpr int kBS = 16;
constexpr int kNK = 64;               // keys per stage
constexpr int kKST = 3;               // K/V ring stages
constexpr int kSoftWarps = 8;          // softmax warps: two per TMEM lane quarter (half a row each)
constexpr int kPrefillThreads = (kSoftWarps + 2) * 32;  // + 1 copy warp, 1 MMA warp
constexpr float kLog2e = 1.4426950408889634f;

// SPLIT: P goes to the tensor cores as hi + lo halves (bf16 keeps 8 bits of a weight;
// the two halves together ~16, as the fp16 path has in one).
template <int D, bool SPLIT> struct PrefillShape {
  static constexpr int DC = D / 64;                  // 64-wide head_dim chunks
  static constexpr int QB = DC * 128 * 128;          // Q tile: [DC][128 rows][64]
  static constexpr int KSB = DC * kNK * 128;         // one stage of K (or V): [DC][NK keys][64]
  static constexpr int PB = (kNK / 64) * 128 * 128;  // P tile: [NK/64][128 rows][64]
  static constexpr int NP = SPLIT ? 2 : 1;           // P tiles per buffer (hi, lo)
  static constexpr int SMEM = 1024 + QB + 2 * kKST * KSB + 2 * NP * PB + 24 * 8 + 16 + 3 * 2 * 128 * 4;
  // TMEM: S double-buffered at columns 0 and NK, the O accumulator at 2 NK.
  static constexpr int COLS = 2 * kNK + D;
  static constexpr int NCOLS = COLS <= 128 ? 128 : (COLS <= 256 ? 256 : 512);
  static constexpr int MIN_BLOCKS = D == 64 ? 2 : 1;
};

struct PrefillParams {
  void* out;
  const void* q;
  const int32_t* cu;
  const int32_t* starts;
  const int32_t* tables;
  const int32_t* seq_rows;
  int32_t* status;
  int64_t out_st, out_sh, q_st, q_sh, table_stride;
  int32_t table_rows, table_cols;
  int32_t group, layer, nbt, q_vec16;
  float scale_log2;
};

// Pipeline (stage i = keys 64 i .. 64 i + 63): the MMA thread issues S(0), then for each
// i: S(i+1) into the other S buffer, then O(i) = P(i) V(i) into O buffer i % 2 once the
// softmax warps stored P(i). The softmax warps turn S(i) into P(i) while the tensor cores
// compute S(i+1) and O(i-1), and fold O(i-1) into their accumulators one stage late.
template <typename T, int D, int TQ>
__global__ void __launch_bounds__(kPrefillThreads, PrefillShape<D, false>::MIN_BLOCKS)
    prefill_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                   const PrefillParams p) {
  constexpr bool kSplit = !Dt<T>::kExactP;
  using S = PrefillShape<D, kSplit>;
  constexpr int DC = S::DC;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + S::QB;                 // [kKST][KSB]
  uint8_t* sV = sK + kKST * S::KSB;         // [kKST][KSB]
  uint8_t* sP = sV + kKST * S::KSB;         // [2][NP][PB]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * S::NP * S::PB);
  uint64_t* kv_full = bars;        // [kKST] TMA bytes landed
  uint64_t* kv_empty = bars + 3;   // [kKST] the stage's MMAs are done with it
  uint64_t* s_full = bars + 6;     // [2] S = Q K^T done
  uint64_t* s_free = bars + 8;     // [2] S read out
  uint64_t* p_full = bars + 10;    // [2] P stored
  uint64_t* o_full = bars + 12;    // [2] O += P(j) V(j) done, j even / odd
  uint64_t* q_ready = bars + 16;   // the softmax warps stored Q
  uint64_t* mma_done = bars + 17;  // every MMA of the CTA has completed (before TMEM is freed)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 24);
  float* s_mx = reinterpret_cast<float*>(bars + 26);  // [2 stage parities][2 halves][128 rows] partial row maxima
  float* s_l = s_mx + 2 * 2 * 128;                    // [2 halves][128 rows] final partial row sums

  const int tile = blockIdx.x, head = blockIdx.y, s = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tok0 = p.cu[s];
  const int n_new = p.cu[s + 1] - tok0;
  if (tile * TQ >= n_new) return;
  const int start = p.starts[s];
  const int rows_here = min(TQ, n_new - tile * TQ);
  const int q_first = start + tile * TQ;  // position of the tile's first query
  int kend = q_first + rows_here;         // keys 0 .. kend-1 are visible to the tile
  if (kend > p.table_cols * kBS) {
    if (tid == 0) report(p.status, PKV_ERR_OUT_OF_RANGE);
    kend = p.table_cols * kBS;
  }
  const int nkb = (kend + kBS - 1) / kBS;
  const int nst = (kend + kNK - 1) / kNK;
  int row = p.seq_rows ? p.seq_rows[s] : s;
  if (row < 0 || row >= p.table_rows) {
    if (tid == 0) report(p.status, PKV_ERR_OUT_OF_RANGE);
    row = -1;
  }
  const int32_t* table = row >= 0 ? p.tables + row * p.table_stride : nullptr;
  const int G = p.group;

  if (tid == 0) {
    for (int i = 0; i < kKST; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], kSoftWarps);
      mbar_init(&p_full[i], kSoftWarps);
      mbar_init(&o_full[i], 1);
    }
    mbar_init(q_ready, kSoftWarps);
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tslot, S::NCOLS);
    tc_fence_before_sync();
  }
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tslot;
  const uint64_t deadline = global_ns() + kWaitBudgetNs;
  auto s_col = [](int b) { return (uint32_t)(b * kNK); };
  constexpr uint32_t kOCol = 2 * kNK;

  if (warp == kSoftWarps) {
    // ---------------------------------------------------------------- TMA copies
    // One copy per lane (a lane issues one (block, tensor, head_dim chunk) of the stage):
    // a single issuing lane cannot keep up with 2 KB copies.
    constexpr int kCopies = (kNK / kBS) * 2 * DC;
    bool ok = true;
    for (int i = 0; i < nst && ok; ++i) {
      const int st = i % kKST;
      if (lane == 0) {
        if (i >= kKST && !mbar_wait_until(&kv_empty[st], ((i / kKST) - 1) & 1, deadline)) {
          report(p.status, PKV_ERR_TIMEOUT);
          ok = false;
        }
        if (ok) mbar_arrive_expect_tx(&kv_full[st], 2 * S::KSB);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (ok && lane < kCopies) {
        const int b = lane / (2 * DC), tensor = (lane / DC) % 2, c = lane % DC;
        const int kb = i * (kNK / kBS) + b;
        // Blocks past the visible keys are masked; the scratch block keeps their rows finite.
        int blk = (kb < nkb && table) ? table[kb] : p.nbt - 1;
        if (blk < 0 || blk >= p.nbt) {
          report(p.status, PKV_ERR_OUT_OF_RANGE);
          blk = p.nbt - 1;
        }
        const int c4 = p.layer * p.nbt + blk;
        uint8_t* dst = (tensor ? sV : sK) + st * S::KSB + c * kNK * 128 + b * kBS * 128;
        tma_load_5d(dst, tensor ? &tmap_v : &tmap_k, 0, 0, c, head, c4, &kv_full[st]);
      }
    }
  } else if (warp == kSoftWarps + 1) {
    // ---------------------------------------------------------------- MMA issue
    if (lane == 0) {
      constexpr bool kBf16 = Dt<T>::code == PKV_BF16;
      constexpr uint32_t idesc_s = umma_idesc_f16(kBf16, false, 128, kNK);
      constexpr uint32_t idesc_o = umma_idesc_f16(kBf16, true, 128, D);
      auto issue_s = [&](int j) -> bool {
        const int st = j % kKST, b = j % 2;
        if (!mbar_wait_until(&kv_full[st], (j / kKST) & 1, deadline)) return false;
        if (j >= 2 && !mbar_wait_until(&s_free[b], ((j / 2) - 1) & 1, deadline)) return false;
        tc_fence_after_sync();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int c = kk / 4, k16 = kk % 4;
          const uint64_t a = umma_desc_sw128(smem_u32(sQ + c * 128 * 128 + k16 * 32), 16, 1024);
          const uint64_t bd = umma_desc_sw128(smem_u32(sK + st * S::KSB + c * kNK * 128 + k16 * 32), 16, 1024);
          umma_f16_ss(tmem + s_col(b), a, bd, idesc_s, kk > 0);
        }
        umma_commit(&s_full[b]);
        return true;
      };
      auto issue_o = [&](int j) -> bool {
        const int st = j % kKST, b = j % 2;
        if (!mbar_wait_until(&p_full[b], (j / 2) & 1, deadline)) return false;
        tc_fence_after_sync();
        uint8_t* pb = sP + b * S::NP * S::PB;
#pragma unroll
        for (int h = 0; h < S::NP; ++h) {
#pragma unroll
          for (int kb = 0; kb < kNK / 16; ++kb) {
            const uint64_t a = umma_desc_sw128(smem_u32(pb + h * S::PB + (kb / 4) * 128 * 128 + (kb % 4) * 32), 16, 1024);
            const uint64_t bd = umma_desc_sw128(smem_u32(sV + st * S::KSB + kb * kBS * 128), kNK * 128, 1024);
            umma_f16_ss(tmem + kOCol, a, bd, idesc_o, j > 0 || h > 0 || kb > 0);
          }
        }
        umma_commit(&o_full[b]);
        umma_commit(&kv_empty[st]);
        return true;
      };
      bool ok = mbar_wait_until(q_ready, 0, deadline) && (nst == 0 || issue_s(0));
      for (int i = 0; i < nst && ok; ++i) {
        ok = (i + 1 >= nst || issue_s(i + 1)) && issue_o(i);
      }
      if (!ok) report(p.status, PKV_ERR_TIMEOUT);
      umma_commit(mma_done);
    }
  } else {
    // ---------------------------------------------------------------- softmax warps: half a row per thread
    // Warps w and w + 4 read TMEM lanes 32 (w % 4) .. + 31: the same rows. Half hf of a row
    // owns keys 32 hf .. 32 hf + 31 of every stage and output columns hf D/2 .. + D/2; the
    // two halves trade their partial maxima through shared memory once per stage.
    constexpr int KH = kNK / 2, DH = D / 2;
    const int hf = warp / 4;
    const int r = (warp % 4) * 32 + lane;  // TMEM lane = tile row
    const int t = r / G, gq = r - t * G;
    const bool valid = r < TQ * G && t < rows_here;
    const int qpos = q_first + t;
    // Q row r (this thread's half of the granules) into the swizzled tile, zeros without a query.
    {
      const T* qrow = reinterpret_cast<const T*>(p.q) + (int64_t)(tok0 + tile * TQ + t) * p.q_st +
                      (int64_t)(head * G + gq) * p.q_sh;
#pragma unroll
      for (int k = 0; k < D / 16; ++k) {
        const int c16 = hf * (D / 16) + k;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (valid) {
          if (p.q_vec16) {
            v = *reinterpret_cast<const uint4*>(qrow + 8 * c16);
          } else {
            const uint32_t* q32 = reinterpret_cast<const uint32_t*>(qrow + 8 * c16);
            v = make_uint4(q32[0], q32[1], q32[2], q32[3]);
          }
        }
        const int c = c16 / 8, gr = c16 % 8;
        *reinterpret_cast<uint4*>(sQ + c * 128 * 128 + r * 128 + ((gr ^ (r & 7)) * 16)) = v;
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(q_ready);

    const uint32_t tl = tmem + ((uint32_t)((warp % 4) * 32) << 16);
    const int pair_bar = 1 + warp % 4;  // named barrier of warps w and w + 4
    // O accumulates in TMEM across stages against a reference max m that moves only when a
    // row's max grows by more than kSlack (in log2 units): weights then stay below 2^kSlack
    // and, in the common case, O needs no rescaling at all. When it does, the warps rescale
    // their rows of O in TMEM after the previous P V completed and before this stage's P is
    // released to the MMA thread. PV(j) completes on o_full[j % 2]; each is confirmed at the
    // start of stage j + 2 (or when a rescale needs it), always before PV(j + 2), the next
    // phase of the same barrier, can be issued: every parity wait is unambiguous.
    constexpr float kSlack = 8.f;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    auto confirm = [&](int j) {  // PV(j) has completed
      if (ok && !mbar_wait_until(&o_full[j % 2], (j / 2) & 1, deadline)) ok = false;
    };
    for (int i = 0; i < nst; ++i) {
      const int b = i % 2;
      // Before P(i) is released, so that PV(i) (the next phase of this barrier) cannot have run.
      if (i >= 2) confirm(i - 2);
      if (ok && !mbar_wait_until(&s_full[b], (i / 2) & 1, deadline)) ok = false;
      tc_fence_after_sync();
      const int key0 = i * kNK + hf * KH;
      uint32_t sa[KH];
      tmem_ld32(tl + s_col(b) + hf * KH, sa);
      tmem_wait_ld();
      tc_fence_before_sync();  // S is in registers: its buffer may take S(i + 2)
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[b]);
      // Raw scores; the max is taken before scaling (the scale is positive). A stage whose
      // every key is visible to every row of the tile needs no mask.
      float mx = -INFINITY;
      if ((i + 1) * kNK - 1 <= q_first && (i + 1) * kNK <= kend) {
#pragma unroll
        for (int e = 0; e < KH; ++e) mx = fmaxf(mx, __uint_as_float(sa[e]));
      } else {
#pragma unroll
        for (int e = 0; e < KH; ++e) {
          const int key = key0 + e;
          if (!(valid && key <= qpos && key < kend)) sa[e] = __float_as_uint(-INFINITY);
          mx = fmaxf(mx, __uint_as_float(sa[e]));
        }
      }
      mx *= p.scale_log2;  // -inf stays -inf
      float* mxb = s_mx + (i % 2) * 256;
      mxb[hf * 128 + r] = mx;
      named_barrier_sync(pair_bar, 64);
      mx = fmaxf(mx, mxb[(1 - hf) * 128 + r]);
      const float m_cand = fmaxf(m, mx);
      float alpha = 1.f;
      if (m_cand - m > kSlack) {  // false while both are -inf (nothing visible yet)
        alpha = ex2(m - m_cand);  // 0 when m was -inf
        m = m_cand;
        l *= alpha;
      }
      if (i > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        confirm(i - 1);
        tc_fence_after_sync();
#pragma unroll
        for (int c = 0; c < DH / 32; ++c) {
          uint32_t ob[32];
          tmem_ld32(tl + kOCol + hf * DH + c * 32, ob);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) ob[e] = __float_as_uint(__uint_as_float(ob[e]) * alpha);
          tmem_st32(tl + kOCol + hf * DH + c * 32, ob);
        }
        tmem_wait_st();
        tc_fence_before_sync();
      }
      const float mref = m == -INFINITY ? 0.f : m;
      float lsum = 0.f;
      uint8_t* pb = sP + b * S::NP * S::PB;
      uint32_t pk[KH / 2], pl[KH / 2];
#pragma unroll
      for (int e = 0; e < KH; e += 2) {
        // ex2(-inf) = 0 for masked keys; every weight is below 2^kSlack
        const float p0 = ex2(fmaf(__uint_as_float(sa[e]), p.scale_log2, -mref));
        const float p1 = ex2(fmaf(__uint_as_float(sa[e + 1]), p.scale_log2, -mref));
        pk[e / 2] = Dt<T>::pack(p0, p1);
        if (kSplit) {
          const float2 hi = Dt<T>::unpack(pk[e / 2]);
          pl[e / 2] = Dt<T>::pack(p0 - hi.x, p1 - hi.y);
        }
        lsum += p0 + p1;
      }
      // keys 32 hf .. 32 hf + 31 of row r: 16-byte granules 4 hf .. 4 hf + 3 of the row
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int gr = hf * 4 + u;
        const int off = (gr / 8) * 128 * 128 + r * 128 + (((gr % 8) ^ (r & 7)) * 16);
        *reinterpret_cast<uint4*>(pb + off) = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        if (kSplit)
          *reinterpret_cast<uint4*>(pb + S::PB + off) = make_uint4(pl[4 * u], pl[4 * u + 1], pl[4 * u + 2], pl[4 * u + 3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[b]);
      l += lsum;  // this half's keys; the halves share the row's reference max
    }
    if (nst >= 2) confirm(nst - 2);
    if (nst >= 1) confirm(nst - 1);
    tc_fence_after_sync();
    float acc[DH];
#pragma unroll
    for (int c = 0; c < DH / 32; ++c) {
      uint32_t ob[32];
      tmem_ld32(tl + kOCol + hf * DH + c * 32, ob);
      tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 32; ++e) acc[c * 32 + e] = __uint_as_float(ob[e]);
    }
    if (!ok) report(p.status, PKV_ERR_TIMEOUT);
    s_l[hf * 128 + r] = l;
    named_barrier_sync(pair_bar, 64);
    l += s_l[(1 - hf) * 128 + r];
    if (valid && ok) {
      const float inv = 1.f / l;
      T* orow = reinterpret_cast<T*>(p.out) + (int64_t)(tok0 + tile * TQ + t) * p.out_st +
                (int64_t)(head * G + gq) * p.out_sh + hf * DH;
#pragma unroll
      for (int e = 0; e < DH; e += 2) *reinterpret_cast<uint32_t*>(orow + e) = Dt<T>::pack(acc[e] * inv, acc[e + 1] * inv);
    }
  }
  __syncthreads();
  if (warp == 0) {
    if (!mbar_wait_until(mma_done, 0, global_ns() + kWaitBudgetNs) && lane == 0) report(p.status, PKV_ERR_TIMEOUT);
    tc_fence_after_sync();
    tmem_dealloc(tmem, S::NCOLS);
  }
}

template <typename T, int D, int TQ>
int launch_prefill(const CUtensorMap& tk, const CUtensorMap& tv, const PrefillParams& p, int max_new, int hkv,
                   int seqs, cudaStream_t st) {
  using S = PrefillShape<D, !Dt<T>::kExactP>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e =
        cudaFuncSetAttribute(prefill_kernel<T, D, TQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM);
    if (e != cudaSuccess) return cuda_status(e);
    configured = true;
  }
  dim3 grid((max_new + TQ - 1) / TQ, hkv, seqs);
  prefill_kernel<T, D, TQ><<<grid, kPrefillThreads, S::SMEM, st>>>(tk, tv, p);
  return launch_status();
}

// Query tokens per CTA: the tile's rows are tokens x group <= 128.
template <typename T, int D>
int launch_group(const CUtensorMap& tk, const CUtensorMap& tv, const PrefillParams& p, int max_new, int hkv,
                 int seqs, cudaStream_t st) {
  return p.group <= 8 ? launch_prefill<T, D, 16>(tk, tv, p, max_new, hkv, seqs, st)
                      : launch_prefill<T, D, 8>(tk, tv, p, max_new, hkv, seqs, st);
}

}  // namespace

}  // namespace pkv

using namespace pkv;

extern "C" int pkv_prefill_attention(const pkv_pool* pool, int32_t layer, const pkv_tables* tables, int32_t num_seqs,
                                     const int32_t* cu_seqlens, const int32_t* starts, int32_t max_new_tokens,
                                     int32_t num_q_heads, void* out, int64_t out_stride_t, int64_t out_stride_h,
                                     const void* q, int64_t q_stride_t, int64_t q_stride_h, float scale,
                                     int32_t* status_dev, pkv_stream_t stream) {
  if (!pool || !tables || !tables->block_tables || !cu_seqlens || !starts || !out || !q)
    return PKV_ERR_INVALID_ARGUMENT;
  if (num_seqs < 0 || num_seqs > 65535 || max_new_tokens < 0 || layer < 0 || layer >= pool->num_layers)
    return PKV_ERR_INVALID_ARGUMENT;
  if (num_seqs == 0 || max_new_tokens == 0) return PKV_OK;
  const int d = pool->head_dim, hkv = pool->num_kv_heads;
  if (pool->block_size != kBS || (d != 64 && d != 128)) return PKV_ERR_UNSUPPORTED;
  if (hkv <= 0 || num_q_heads <= 0 || num_q_heads % hkv != 0) return PKV_ERR_INVALID_ARGUMENT;
  const int group = num_q_heads / hkv;
  if (group > 16) return PKV_ERR_UNSUPPORTED;
  if (tables->cols <= 0 || tables->rows <= 0 || (!tables->seq_rows && tables->rows < num_seqs))
    return PKV_ERR_INVALID_ARGUMENT;
  auto aligned4 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 3) == 0; };
  if (!aligned4(q) || !aligned4(out) || ((q_stride_t | q_stride_h | out_stride_t | out_stride_h) & 1))
    return PKV_ERR_INVALID_ARGUMENT;
  CUtensorMap tk, tv;
  if (!get_pool_maps(*pool, &tk, &tv, 1, 1)) return PKV_ERR_CUDA;  // one head, one 64-wide chunk per copy
  PrefillParams p{};
  p.out = out;
  p.q = q;
  p.cu = cu_seqlens;
  p.starts = starts;
  p.tables = tables->block_tables;
  p.seq_rows = tables->seq_rows;
  p.status = status_dev;
  p.out_st = out_stride_t;
  p.out_sh = out_stride_h;
  p.q_st = q_stride_t;
  p.q_sh = q_stride_h;
  p.table_stride = tables->stride;
  p.table_rows = tables->rows;
  p.table_cols = tables->cols;
  p.group = group;
  p.layer = layer;
  p.nbt = pool->num_blocks_total;
  p.scale_log2 = scale * kLog2e;
  p.q_vec16 = (reinterpret_cast<uintptr_t>(q) & 15) == 0 && ((q_stride_t | q_stride_h) & 7) == 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (pool->dtype == PKV_F16)
    return d == 64 ? launch_group<__half, 64>(tk, tv, p, max_new_tokens, hkv, num_seqs, st)
                   : launch_group<__half, 128>(tk, tv, p, max_new_tokens, hkv, num_seqs, st);
  if (pool->dtype == PKV_BF16)
    return d == 64 ? launch_group<__nv_bfloat16, 64>(tk, tv, p, max_new_tokens, hkv, num_seqs, st)
                   : launch_group<__nv_bfloat16, 128>(tk, tv, p, max_new_tokens, hkv, num_seqs, st);
  return PKV_ERR_UNSUPPORTED;
}
