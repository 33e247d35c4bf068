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
// query heads (18 x 7 = 126 rows for Qwen2's group of 7), so every K/V block read
// serves the whole group. Keys stream in stages of NK = 64 (four blocks) through TMA
// rings with separate K and V stages: S = Q K^T (M 128 x N 64, fp32 in TMEM) frees its K
// stage as soon as it completes, P V frees the V stage, so a K copy has two to three
// stages of softmax time to land instead of one. Eight softmax warps (half a row per
// thread) turn S into P, written to shared memory as fp16/bf16, and O += P V
// accumulates in TMEM against a lazily moved reference max. One warp issues the TMA
// copies (block ids looked up 32 at a time, ahead of use), one thread the MMAs;
// mbarriers (MMA completion through tcgen05.commit) order the three roles. Only the
// causal part of each sequence is visited; keys past a tile's last position are masked
// to -inf.
#include <algorithm>

#include "common.cuh"
#include "tcgen05.cuh"

namespace pkv {
namespace {

constexpr int kBS = 16;
constexpr int kNK = 64;                      // keys per stage
constexpr int kKS = 4;                       // K ring stages (freed when S = Q K^T completes)
constexpr int kVS = 4;                       // V ring stages (freed when O += P V completes)
constexpr int kBars = 2 * (kKS + kVS) + 4;   // + p_full (2), q_ready, mma_done
constexpr int kMaxSeqs = 2048;               // sequences per launch (the host splits larger packs)
constexpr float kLog2e = 1.4426950408889634f;

// SPLIT: P goes to the tensor cores as hi + lo halves (bf16 keeps 8 bits of a weight;
// the two halves together ~16, as the fp16 path has in one).
template <int D, bool SPLIT> struct PrefillShape {
  static constexpr int DC = D / 64;                  // 64-wide head_dim chunks
  static constexpr int KSB = DC * kNK * 128;         // one stage of K (or V): [DC][NK keys][64], 128B-swizzled
  static constexpr int QB = DC * 128 * 128;          // Q tile in shared memory: [DC][128 rows][64]
  // TMEM columns: two S buffers at 0 and NK, O at 2 NK, then Q (packed 16-bit pairs, when
  // it fits). P(j) is written over S(j) in S(j)'s own buffer (32 columns of packed pairs;
  // bf16 adds its lo half in the next 32). At head_dim 64 with bf16, Q stays in shared
  // memory.
  static constexpr bool QT = !(SPLIT && D == 64);
  static constexpr int OCOL = 2 * kNK;
  static constexpr int QCOL = OCOL + D;
  static constexpr int COLS = QCOL + (QT ? D / 2 : 0);
  static constexpr int NCOLS = COLS <= 128 ? 128 : (COLS <= 256 ? 256 : 512);
  static constexpr int MIN_BLOCKS = NCOLS <= 256 ? 2 : 1;
  // Softmax warps: one per TMEM lane quarter (a whole row per thread) when two CTAs share an
  // SM, else two per quarter (half a row each) so that an SM still runs eight.
  static constexpr int SW = MIN_BLOCKS == 2 ? 4 : 8;
  static constexpr int HALVES = SW / 4;
  static constexpr int THREADS = (SW + 2) * 32;  // + 1 copy warp, 1 MMA warp
  static constexpr int SMEM = 1024 + (QT ? 0 : QB) + (kKS + kVS) * KSB + (kBars + 2) * 8 + 3 * 2 * 128 * 4 +
                              (kMaxSeqs + 1) * 4;  // + tiles before each sequence
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
  int32_t group, layer, nbt, q_vec16, out_vec16;
  int32_t num_seqs, seq_base, hkv;  // sequences of this launch; table row = seq_base + s without seq_rows
  float scale_log2;
};

// Pipeline (stage i = keys 64 i .. 64 i + 63). The MMA thread issues S(0) and S(1), then
// for each i, once the softmax warps stored P(i): O += P(i) V(i), then (after that MMA
// completed) S(i+2) = Q K(i+2)^T into the buffer that held S(i) and P(i). The softmax warps
// turn S(i) into P(i) in place, in S(i)'s buffer, while the tensor cores compute O(i-1)
// and S(i+1): P(i) never waits for O(i-1), which reads P(i-1) from the other buffer. P (and
// Q where it fits) is the A operand straight from TMEM, so most MMAs read only K or V from
// shared memory. An MMA burst costs several hundred cycles to issue however small it is
// (measured), which is why each stage has one burst rather than two.
template <typename T, int D, int TQ>
__global__ void __launch_bounds__(PrefillShape<D, !Dt<T>::kExactP>::THREADS, PrefillShape<D, !Dt<T>::kExactP>::MIN_BLOCKS)
    prefill_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                   const PrefillParams p) {
  constexpr bool kSplit = !Dt<T>::kExactP;
  using S = PrefillShape<D, kSplit>;
  constexpr int DC = S::DC;
  constexpr bool kQT = S::QT;
  constexpr int SW = S::SW, HALVES = S::HALVES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                        // [QB] when Q is not in TMEM
  uint8_t* sK = sQ + (kQT ? 0 : S::QB);      // [kKS][KSB]
  uint8_t* sV = sK + kKS * S::KSB;           // [kVS][KSB]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kVS * S::KSB);
  uint64_t* k_full = bars;                   // [kKS] TMA bytes of K landed
  uint64_t* v_full = k_full + kKS;           // [kVS] TMA bytes of V landed
  // One commit per MMA group: S(j) done tells the softmax warps that S(j) is ready and the
  // copy warp that K stage j % kKS is free; O(j) done frees V stage j % kVS (and O).
  uint64_t* s_done = v_full + kVS;           // [kKS] S(j) = Q K(j)^T done, j % kKS
  uint64_t* o_done = s_done + kKS;           // [kVS] O += P(j) V(j) done, j % kVS
  uint64_t* p_full = o_done + kVS;           // [2] P(j) stored in TMEM, j even / odd
  uint64_t* q_ready = p_full + 2;            // the softmax warps stored Q
  uint64_t* mma_done = q_ready + 1;          // every MMA of the CTA has completed (before TMEM is freed)
  static_assert(kBars == 2 * (kKS + kVS) + 4, "barrier layout");
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + kBars);
  float* s_mx = reinterpret_cast<float*>(bars + kBars + 2);  // [2 stage parities][2 halves][128 rows] partial row maxima
  float* s_l = s_mx + 2 * 2 * 128;                           // [2 halves][128 rows] final partial row sums

  int* sTiles = reinterpret_cast<int*>(s_l + 2 * 128);  // [num_seqs + 1] tiles before sequence s
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int B = p.num_seqs, G = p.group;
  if (warp == SW) {  // tiles per sequence, prefix-summed (a sequence without new tokens has none)
    int carry = 0;
    for (int base = 0; base < B; base += 32) {
      const int i = base + lane;
      const int n = i < B ? p.cu[i + 1] - p.cu[i] : 0;
      int inc = n > 0 ? (n + TQ - 1) / TQ : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {  // inclusive warp scan
        const int u = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += u;
      }
      if (i < B) sTiles[i + 1] = carry + inc;
      carry += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (lane == 0) sTiles[0] = 0;
  }
  if (tid == 0) {
    for (int i = 0; i < kKS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&s_done[i], 1);
    }
    for (int i = 0; i < kVS; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&o_done[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_full[i], SW);
    }
    mbar_init(q_ready, SW);
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

  // Work items: (sequence, 16-18-token tile, KV head), heads fastest; CTA g takes items g,
  // g + gridDim.x, ... Every role walks the same items and numbers stages across them
  // (stage j of the CTA = its item's stage j - base), so ring slots and barrier parities
  // simply continue from one item to the next.
  const int n_items = sTiles[B] * p.hkv;
  struct Item {
    int s, head, tile, tok0, n_new, start, rows_here, q_first, kend, nkb, nst;
    const int32_t* table;
  };
  auto item_at = [&](int w) {
    Item it;
    it.head = w % p.hkv;
    const int tw = w / p.hkv;
    int lo = 0, hi = B - 1;  // the largest s with sTiles[s] <= tw: the sequence holding tile tw
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (sTiles[mid] <= tw) lo = mid; else hi = mid - 1;
    }
    it.s = lo;
    it.tile = tw - sTiles[lo];
    it.tok0 = p.cu[lo];
    it.n_new = p.cu[lo + 1] - it.tok0;
    it.start = p.starts[lo];
    it.rows_here = min(TQ, it.n_new - it.tile * TQ);
    it.q_first = it.start + it.tile * TQ;  // position of the tile's first query
    it.kend = it.q_first + it.rows_here;   // keys 0 .. kend-1 are visible to the tile
    if (it.kend > p.table_cols * kBS) {
      if (lane == 0) report(p.status, PKV_ERR_OUT_OF_RANGE);
      it.kend = p.table_cols * kBS;
    }
    it.nkb = (it.kend + kBS - 1) / kBS;
    it.nst = (it.kend + kNK - 1) / kNK;
    int row = p.seq_rows ? p.seq_rows[lo] : p.seq_base + lo;
    if (row < 0 || row >= p.table_rows) {
      if (lane == 0) report(p.status, PKV_ERR_OUT_OF_RANGE);
      row = -1;
    }
    it.table = row >= 0 ? p.tables + (int64_t)row * p.table_stride : nullptr;
    return it;
  };

  if (warp == SW) {
    // ---------------------------------------------------------------- TMA copies
    // One copy per lane (lane l < kCopies copies head_dim chunk l % DC of block l / DC of the
    // stage; a single issuing lane cannot keep up with 2 KB copies), K of a stage as soon as
    // its K stage is free, then V. Block ids come from a window of 32 looked up at once,
    // the next window in flight meanwhile.
    constexpr int kCopies = (kNK / kBS) * DC;
    constexpr int kStagesPerWindow = 32 / (kNK / kBS);
    const int b = lane / DC, c = lane % DC;
    bool ok = true;
    int gs = 0;  // stages of earlier items
    for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x) {
    const Item it = item_at(w);
    const int nst = it.nst, nkb = it.nkb, head = it.head;
    const int32_t* table = it.table;
    auto lookup = [&](int kb) -> int {
      // Blocks past the visible keys are masked; the scratch block keeps their rows finite.
      int blk = (kb < nkb && table) ? table[kb] : p.nbt - 1;
      if (blk < 0 || blk >= p.nbt) {
        report(p.status, PKV_ERR_OUT_OF_RANGE);
        blk = p.nbt - 1;
      }
      return blk;
    };
    int win = lookup(lane), win_next = lookup(32 + lane);
    for (int i = 0; i < nst && ok; ++i) {
      if (i > 0 && i % kStagesPerWindow == 0) {
        win = win_next;
        win_next = lookup(32 * (i / kStagesPerWindow + 1) + lane);
      }
      const int blk = __shfl_sync(0xffffffffu, win, (i * (kNK / kBS) + b) % 32);
      const int c4 = p.layer * p.nbt + blk;
      const int j = gs + i;  // the CTA's stage
      const int sk = j % kKS, sv = j % kVS;
      if (lane == 0) {
        if (j >= kKS && !mbar_wait_until(&s_done[sk], ((j / kKS) - 1) & 1, deadline)) {
          report(p.status, PKV_ERR_TIMEOUT);
          ok = false;
        }
        if (ok) mbar_arrive_expect_tx(&k_full[sk], S::KSB);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (ok && lane < kCopies)
        tma_load_5d(sK + sk * S::KSB + c * kNK * 128 + b * kBS * 128, &tmap_k, 0, 0, c, head, c4, &k_full[sk]);
      if (lane == 0 && ok) {
        if (j >= kVS && !mbar_wait_until(&o_done[sv], ((j / kVS) - 1) & 1, deadline)) {
          report(p.status, PKV_ERR_TIMEOUT);
          ok = false;
        }
        if (ok) mbar_arrive_expect_tx(&v_full[sv], S::KSB);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (ok && lane < kCopies)
        tma_load_5d(sV + sv * S::KSB + c * kNK * 128 + b * kBS * 128, &tmap_v, 0, 0, c, head, c4, &v_full[sv]);
    }
    gs += nst;
    }
  } else if (warp == SW + 1) {
    // ---------------------------------------------------------------- MMA issue
    if (lane == 0) {
      constexpr bool kBf16 = Dt<T>::code == PKV_BF16;
      constexpr uint32_t idesc_s = umma_idesc_f16(kBf16, false, 128, kNK);
      constexpr uint32_t idesc_o = umma_idesc_f16(kBf16, true, 128, D);
      constexpr int NP = kSplit ? 2 : 1;  // P as hi + lo halves for bf16
      // Descriptors of a group are computed before its barrier waits and pinned there, so
      // the MMAs of a group issue back to back (a probe measured ~45 cycles per MMA that way
      // against ~120 with each descriptor computed just before its MMA).
      auto pin = [](uint64_t& x) { asm volatile("" : "+l"(x)); };
      auto issue_s = [&](int j, bool after_o) -> bool {  // S(j) into buffer j % 2, over P(j - 2)
        const int st = j % kKS, b = j % 2;
        uint64_t bk[D / 16], aq[D / 16];
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int c = kk / 4, k16 = kk % 4;
          bk[kk] = umma_desc_sw128(smem_u32(sK + st * S::KSB + c * kNK * 128 + k16 * 32), 16, 1024);
          aq[kk] = kQT ? 0 : umma_desc_sw128(smem_u32(sQ + c * 128 * 128 + k16 * 32), 16, 1024);
          pin(bk[kk]);
          pin(aq[kk]);
        }
        if (!mbar_wait_until(&k_full[st], (j / kKS) & 1, deadline)) return false;
        // Within an item, P(j - 2) lives in this buffer until O(j - 2) has read it.
        if (after_o && !mbar_wait_until(&o_done[(j - 2) % kVS], ((j - 2) / kVS) & 1, deadline)) return false;
        tc_fence_after_sync();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          if (kQT) {
            umma_f16_ts(tmem + s_col(b), tmem + S::QCOL + kk * 8, bk[kk], idesc_s, kk > 0);
          } else {
            umma_f16_ss(tmem + s_col(b), aq[kk], bk[kk], idesc_s, kk > 0);
          }
        }
        umma_commit(&s_done[st]);
        return true;
      };
      auto issue_o = [&](int j, bool first) -> bool {  // first: the item's first stage overwrites O
        const int st = j % kVS, b = j % 2;
        uint64_t bv[kNK / 16];
#pragma unroll
        for (int kb = 0; kb < kNK / 16; ++kb) {
          bv[kb] = umma_desc_sw128(smem_u32(sV + st * S::KSB + kb * kBS * 128), kNK * 128, 1024);
          pin(bv[kb]);
        }
        if (!mbar_wait_until(&p_full[b], (j / 2) & 1, deadline)) return false;
        if (!mbar_wait_until(&v_full[st], (j / kVS) & 1, deadline)) return false;
        tc_fence_after_sync();
#pragma unroll
        for (int h = 0; h < NP; ++h) {
#pragma unroll
          for (int kb = 0; kb < kNK / 16; ++kb)
            umma_f16_ts(tmem + S::OCOL, tmem + s_col(b) + h * (kNK / 2) + kb * 8, bv[kb], idesc_o,
                        !first || h > 0 || kb > 0);
        }
        umma_commit(&o_done[st]);
        return true;
      };
      // S(j + 2) overwrites P(j) once O(j) has read it. q_ready(k) comes after the softmax
      // warps read item k - 1's O (so every O of that item completed) and waited for all its
      // S: item k's first two S and its O-overwriting first P V may go.
      bool ok = true;
      int gs = 0, k = 0;
      for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x, ++k) {
        const int nst = item_at(w).nst;
        ok = mbar_wait_until(q_ready, k & 1, deadline) && issue_s(gs, false) && (nst < 2 || issue_s(gs + 1, false));
        for (int i = 0; i < nst && ok; ++i)
          ok = issue_o(gs + i, i == 0) && (i + 2 >= nst || issue_s(gs + i + 2, true));
        gs += nst;
      }
      if (!ok) report(p.status, PKV_ERR_TIMEOUT);
      if (k > 0) umma_commit(mma_done); else mbar_arrive(mma_done);
    }
  } else {
    // ---------------------------------------------------------------- softmax warps
    // Warp w reads TMEM lanes 32 (w % 4) .. + 31: tile rows. With two warps per lane quarter
    // (HALVES = 2), half hf = w / 4 of a row owns keys KH hf .. KH hf + KH - 1 of every stage
    // and output columns DH hf .. + DH - 1, and the two halves trade their partial maxima
    // through shared memory once per stage; with one, a thread owns its whole row.
    constexpr int KH = kNK / HALVES, DH = D / HALVES;
    const int hf = warp / 4;
    const int r = (warp % 4) * 32 + lane;  // TMEM lane = tile row
    const int t = r / G, gq = r - t * G;
    const uint32_t tl = tmem + ((uint32_t)((warp % 4) * 32) << 16);
    const int pair_bar = 1 + warp % 4;  // named barrier of warps w and w + 4
    // O accumulates in TMEM across stages against a reference max m that moves only when a
    // row's max grows by more than kSlack (in log2 units): weights then stay below 2^kSlack
    // and, in the common case, O needs no rescaling at all. When it does, the warps rescale
    // their rows of O in TMEM after the previous P V completed and before this stage's P is
    // released to the MMA thread. Parity waits stay unambiguous: S(j + kKS) cannot be issued
    // before P(j + kKS - 2) exists, and the softmax warps wait for O(j) only before P(j + 1)
    // is released (or, for an item's last stage, before reading O), when O(j + kVS) cannot
    // have been issued.
    constexpr float kSlack = 8.f;
    bool ok = true;
    auto confirm = [&](int j) {  // PV(j) has completed
      if (ok && !mbar_wait_until(&o_done[j % kVS], (j / kVS) & 1, deadline)) ok = false;
    };
    int gs = 0;  // stages of earlier items
    for (int w = blockIdx.x; w < n_items; w += gridDim.x) {
    const Item it = item_at(w);
    const int nst = it.nst, q_first = it.q_first, kend = it.kend, tok0 = it.tok0, tile = it.tile, head = it.head;
    const bool valid = r < TQ * G && t < it.rows_here;
    const int qpos = q_first + t;
    // Q row r, this thread's half of head_dim, as the S MMAs' A operand: into TMEM (packed
    // 16-bit pairs) or into the swizzled shared-memory tile; zeros for rows without a query.
    {
      const T* qrow = reinterpret_cast<const T*>(p.q) + (int64_t)(tok0 + tile * TQ + t) * p.q_st +
                      (int64_t)(head * G + gq) * p.q_sh + hf * DH;
#pragma unroll
      for (int c = 0; c < DH / 32; ++c) {  // 32 elements = 16 columns = 4 granules of 16 bytes
        uint32_t qv[16];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          uint4 v = make_uint4(0, 0, 0, 0);
          if (valid) {
            if (p.q_vec16) {
              v = *reinterpret_cast<const uint4*>(qrow + c * 32 + 8 * k);
            } else {
              const uint32_t* q32 = reinterpret_cast<const uint32_t*>(qrow + c * 32 + 8 * k);
              v = make_uint4(q32[0], q32[1], q32[2], q32[3]);
            }
          }
          if (kQT) {
            qv[4 * k] = v.x, qv[4 * k + 1] = v.y, qv[4 * k + 2] = v.z, qv[4 * k + 3] = v.w;
          } else {
            const int c16 = (hf * DH + c * 32) / 8 + k;  // granule of the row
            const int cc = c16 / 8, gr = c16 % 8;
            *reinterpret_cast<uint4*>(sQ + cc * 128 * 128 + r * 128 + ((gr ^ (r & 7)) * 16)) = v;
          }
        }
        if (kQT) tmem_st16(tl + S::QCOL + hf * (DH / 2) + c * 16, qv);
      }
    }
    if (!kQT) fence_proxy_async_smem();
    tmem_wait_st();
    tc_fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(q_ready);

    float m = -INFINITY, l = 0.f;
    for (int i = 0; i < nst; ++i) {
      const int j = gs + i;  // the CTA's stage
      const int b = j % 2;
      if (ok && !mbar_wait_until(&s_done[j % kKS], (j / kKS) & 1, deadline)) ok = false;
      tc_fence_after_sync();
      const int key0 = i * kNK + hf * KH;
      uint32_t sa[KH];
#pragma unroll
      for (int c = 0; c < KH / 32; ++c) tmem_ld32(tl + s_col(b) + hf * KH + c * 32, *reinterpret_cast<uint32_t(*)[32]>(sa + c * 32));
      tmem_wait_ld();
      // Raw scores; the max is taken before scaling (the scale is positive). A stage whose
      // every key is visible to every row of the tile needs no mask.
      if (!((i + 1) * kNK - 1 <= q_first && (i + 1) * kNK <= kend)) {
#pragma unroll
        for (int e = 0; e < KH; ++e) {
          const int key = key0 + e;
          if (!(valid && key <= qpos && key < kend)) sa[e] = __float_as_uint(-INFINITY);
        }
      }
      float mt[KH / 2];
#pragma unroll
      for (int e = 0; e < KH / 2; ++e) mt[e] = fmaxf(__uint_as_float(sa[e]), __uint_as_float(sa[e + KH / 2]));
#pragma unroll
      for (int w = KH / 4; w > 0; w >>= 1) {
#pragma unroll
        for (int e = 0; e < w; ++e) mt[e] = fmaxf(mt[e], mt[e + w]);
      }
      float mx = mt[0] * p.scale_log2;  // -inf stays -inf
      if (HALVES == 2) {
        float* mxb = s_mx + (j % 2) * 256;
        mxb[hf * 128 + r] = mx;
        named_barrier_sync(pair_bar, 64);
        mx = fmaxf(mx, mxb[(1 - hf) * 128 + r]);
      }
      const float m_cand = fmaxf(m, mx);
      float alpha = 1.f;
      if (m_cand - m > kSlack) {  // false while both are -inf (nothing visible yet)
        alpha = ex2(m - m_cand);  // 0 when m was -inf
        m = m_cand;
        l *= alpha;
      }
      if (i > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        confirm(j - 1);
        tc_fence_after_sync();
#pragma unroll
        for (int c = 0; c < DH / 32; ++c) {
          uint32_t ob[32];
          tmem_ld32(tl + S::OCOL + hf * DH + c * 32, ob);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) ob[e] = __float_as_uint(__uint_as_float(ob[e]) * alpha);
          tmem_st32(tl + S::OCOL + hf * DH + c * 32, ob);
        }
      }
      const float mref = m == -INFINITY ? 0.f : m;
      float2 lsum[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};  // independent paired chains
      const float2 scale2 = make_float2(p.scale_log2, p.scale_log2), negm2 = make_float2(-mref, -mref);
      uint32_t pk[KH / 2], pl[KH / 2];
#pragma unroll
      for (int e = 0; e < KH; e += 2) {
        // ex2(-inf) = 0 for masked keys; every weight is below 2^kSlack
        const float2 x = ffma2(make_float2(__uint_as_float(sa[e]), __uint_as_float(sa[e + 1])), scale2, negm2);
        const float p0 = ex2(x.x), p1 = ex2(x.y);
        pk[e / 2] = Dt<T>::pack(p0, p1);
        if (kSplit) {
          const float2 hi = Dt<T>::unpack(pk[e / 2]);
          pl[e / 2] = Dt<T>::pack(p0 - hi.x, p1 - hi.y);
        }
        lsum[(e / 2) % 2] = fadd2(lsum[(e / 2) % 2], make_float2(p0, p1));
      }
      // P(i) goes over S(i), in its buffer: keys KH hf .. + KH - 1 are packed columns
      // KH / 2 hf .. + KH / 2 - 1 (lo half NK / 2 further). This thread's S loads completed
      // above and, with two halves per row, the pair barrier ordered the other half's too;
      // O(i - 2), which read the buffer's previous P, completed before S(i) was written.
      tc_fence_after_sync();
#pragma unroll
      for (int c = 0; c < KH / 32; ++c) {
        tmem_st16(tl + s_col(b) + hf * (KH / 2) + c * 16, *reinterpret_cast<const uint32_t(*)[16]>(pk + c * 16));
        if (kSplit)
          tmem_st16(tl + s_col(b) + kNK / 2 + hf * (KH / 2) + c * 16,
                    *reinterpret_cast<const uint32_t(*)[16]>(pl + c * 16));
      }
      tmem_wait_st();
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[b]);
      l += (lsum[0].x + lsum[1].x) + (lsum[0].y + lsum[1].y);  // this thread's keys; halves share the reference max
    }
    confirm(gs + nst - 1);  // nst >= 1; the commit of this PV tracks every earlier MMA as well
    tc_fence_after_sync();
    float acc[DH];
#pragma unroll
    for (int c = 0; c < DH / 32; ++c) {
      uint32_t ob[32];
      tmem_ld32(tl + S::OCOL + hf * DH + c * 32, ob);
      tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 32; ++e) acc[c * 32 + e] = __uint_as_float(ob[e]);
    }
    if (!ok) report(p.status, PKV_ERR_TIMEOUT);
    if (HALVES == 2) {
      s_l[hf * 128 + r] = l;
      named_barrier_sync(pair_bar, 64);
      l += s_l[(1 - hf) * 128 + r];
    }
    if (valid && ok) {
      const float inv = 1.f / l;
      T* orow = reinterpret_cast<T*>(p.out) + (int64_t)(tok0 + tile * TQ + t) * p.out_st +
                (int64_t)(head * G + gq) * p.out_sh + hf * DH;
      if (p.out_vec16) {
#pragma unroll
        for (int e = 0; e < DH; e += 8)
          *reinterpret_cast<uint4*>(orow + e) =
              make_uint4(Dt<T>::pack(acc[e] * inv, acc[e + 1] * inv), Dt<T>::pack(acc[e + 2] * inv, acc[e + 3] * inv),
                         Dt<T>::pack(acc[e + 4] * inv, acc[e + 5] * inv), Dt<T>::pack(acc[e + 6] * inv, acc[e + 7] * inv));
      } else {
#pragma unroll
        for (int e = 0; e < DH; e += 2) *reinterpret_cast<uint32_t*>(orow + e) = Dt<T>::pack(acc[e] * inv, acc[e + 1] * inv);
      }
    }
    gs += nst;
    }  // items
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
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return cuda_status(e);
  // Persistent CTAs: as many as are resident at once, or as many items as there can be.
  // The work split is read from cu_seqlens on the device, kMaxSeqs sequences per launch.
  for (int s0 = 0; s0 < seqs; s0 += kMaxSeqs) {
    PrefillParams q = p;
    q.num_seqs = min(kMaxSeqs, seqs - s0);
    q.cu = p.cu + s0;
    q.starts = p.starts + s0;
    q.seq_base = s0;
    if (p.seq_rows) q.seq_rows = p.seq_rows + s0;
    const int64_t items = (int64_t)q.num_seqs * ((max_new + TQ - 1) / TQ) * hkv;
    const int grid = (int)std::min<int64_t>(items, (int64_t)sms * S::MIN_BLOCKS);
    prefill_kernel<T, D, TQ><<<grid, S::THREADS, S::SMEM, st>>>(tk, tv, q);
    const int rc = launch_status();
    if (rc != PKV_OK) return rc;
  }
  return PKV_OK;
}

// Query tokens per CTA: the tile's rows are tokens x group <= 128.
template <typename T, int D>
int launch_group(const CUtensorMap& tk, const CUtensorMap& tv, const PrefillParams& p, int max_new, int hkv,
                 int seqs, cudaStream_t st) {
  // As many tokens as fill the 128 rows: 18 x 7 = 126 for Qwen2's group of 7 (16 tokens
  // would leave 16 rows idle), 16 x 8, 8 x 9..16.
  if (p.group == 7) return launch_prefill<T, D, 18>(tk, tv, p, max_new, hkv, seqs, st);
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
  p.hkv = hkv;
  p.num_seqs = num_seqs;
  p.seq_base = 0;
  p.q_vec16 = (reinterpret_cast<uintptr_t>(q) & 15) == 0 && ((q_stride_t | q_stride_h) & 7) == 0;
  p.out_vec16 = (reinterpret_cast<uintptr_t>(out) & 15) == 0 && ((out_stride_t | out_stride_h) & 7) == 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (pool->dtype == PKV_F16)
    return d == 64 ? launch_group<__half, 64>(tk, tv, p, max_new_tokens, hkv, num_seqs, st)
                   : launch_group<__half, 128>(tk, tv, p, max_new_tokens, hkv, num_seqs, st);
  if (pool->dtype == PKV_BF16)
    return d == 64 ? launch_group<__nv_bfloat16, 64>(tk, tv, p, max_new_tokens, hkv, num_seqs, st)
                   : launch_group<__nv_bfloat16, 128>(tk, tv, p, max_new_tokens, hkv, num_seqs, st);
  return PKV_ERR_UNSUPPORTED;
}
