// Paged decode attention for sm_100a, fused with the one-token KV append.
//
// Replaces, per layer and decode step, PagedDecodeContext.attend
// (engine/kv_cache.py:611-620): the index_put append, the gather of every
// sequence's blocks into a padded contiguous copy, and decode_attention's SDPA
// (engine/model.py:126-147). Here nothing is gathered: K/V blocks are read in
// place through the block table, each exactly once, straight into shared memory.
//
// Work split. A CTA streams an ordered list of segments, each a run of consecutive
// blocks of one sequence. Every CTA derives the split from context_lens in its prologue
// (which, with PKV_DECODE_INPUTS_READY, runs before it waits for the previous kernel),
// by one of two rules:
//  * long ranges (at least kFlatMin blocks per CTA on average): the batch's blocks are
//    laid end to end and cut into equal ranges of ceil(T / C) blocks, one per CTA (T
//    blocks, C CTAs). Every CTA streams the same bytes whatever the mix of lengths; its
//    range covers the tail of one sequence, whole sequences and the head of another, and
//    holds at most two cut pieces (its first and its last).
//  * short ranges: sequences longer than a cap are cut into ceil(n / cap) balanced chunks,
//    and CTA g takes units g, g + C, ... The cap is max(kMinCap, ceil(T / max(C - I,
//    C / 4))) (I: sequences), which fits all units in one wave when the batch allows; for
//    batches of more than C / 2 sequences, the smallest of a fixed list of candidates
//    (12 .. 64 blocks) whose units fill at most 29 / 32 of the CTAs, where one does. Units then
//    differ in length, and the CTAs that finish early make room for the next launch's
//    CTAs, which fill their rings while this launch ends; with equal ranges every CTA
//    would end at once and nothing of the next launch could start early (measured slower
//    at 64 sequences of 128..2048 tokens, faster at 8..32 K tokens).
// A sequence cut into several segments leaves one partial softmax state per segment; the
// CTA that takes the sequence's last ticket merges them in segment order, so the result
// does not depend on which CTA came last.
//
// Inside a CTA one producer warp resolves block ids through the block table (32 at a
// time, one lookup per lane, the next 32 in flight) and keeps a ring of stages full
// with TMA copies of a block's K and V for all KV heads at once (adjacent in the pool;
// 128B swizzle, L2 evict-first); kIssueLanes lanes issue the copies of consecutive
// blocks with one instruction. The 8 consumer warps split the KV heads
// (8 / Hkv warps per head); the CTA's j-th block goes, for every head, to warp
// j % (8 / Hkv) of that head through stage j % S (S a multiple of 8 / Hkv), so each warp
// waits on every phase of its stages in turn (an mbarrier parity wait cannot tell a
// phase from the one two later). Each consumer runs the 16-key flash step on mma.sync
// m16n8k16 with the M = 16 rows being its head's GQA group of query heads (the reference
// regroups head h to (h / group, h % group) the same way), so a tile read from HBM serves
// the whole group (attn_tile.cuh). At the end of a segment the warps of a head merge
// their softmax states through shared memory and write the output (a whole sequence) or
// the segment's partial state.
#include <algorithm>
#include <cstdlib>

#include "attn_tile.cuh"
#include "common.cuh"

namespace pkv {
namespace {

constexpr int kBS = 16;  // tokens per block handled by this kernel
constexpr int kNC = 8;   // consumer warps
constexpr int kThreads = (kNC + 1) * 32;
constexpr int kMaxBatch = 1024;    // the per-sequence tables live in shared memory
constexpr int kSmallBatch = 256;   // batches up to this size take tables a quarter as large
constexpr int kMinCap = 12;        // chunks: the fallback rule never cuts sequences of up to 12 blocks
// Chunk caps (blocks) the split tries, smallest first, for batches of more than C / 2
// sequences: it takes the smallest whose units fill at most 29/32 of the C CTAs, so that
// every unit starts in the first wave and the longest units stay short, while a few CTAs
// are left to the next launch's ring fill. (The fallback rule divides by C - I, which such
// batches make small, so its cap grows far beyond what fills the CTAs.)
constexpr int kNumCaps = 16;
__host__ __device__ constexpr int cap_candidate(int k) {
  constexpr int caps[kNumCaps] = {12, 13, 14, 15, 16, 18, 20, 22, 24, 26, 28, 32, 36, 40, 48, 64};
  return caps[k];
}
constexpr int kFlatMin = 128;      // blocks per CTA from which the ranges are equal
constexpr int kMinQuota = 4;       // equal ranges: never fewer blocks per CTA than this
constexpr int kIssueLanes = 4;     // producer lanes issuing copies together
constexpr int kMergeBatch = 4;     // segment states a merging thread loads at once
constexpr int kMaxPending = 32;    // cut segments of one CTA whose tickets are taken at the end
constexpr int kTicketBatch = 8;    // tickets thread 0 keeps in flight at once
constexpr float kLog2e = 1.4426950408889634f;

// Stages per consumer warp for `fixed` bytes of shared memory besides the ring: two CTAs
// per SM when each warp keeps 2+ stages in half the shared memory and the fragments of 8
// rows fit half the registers, else one CTA with up to 4 stages per warp.
constexpr bool ring_two(int fixed, int stage, int wph, int rk) {
  return (113 * 1024 - fixed) / (2 * stage * wph) >= 2 && rk <= 8;
}
constexpr int ring_pw(int fixed, int stage, int wph, int rk) {
  return ring_two(fixed, stage, wph, rk) ? std::min((113 * 1024 - fixed) / (2 * stage * wph), 3)
                                         : std::min((226 * 1024 - fixed) / (2 * stage * wph), 4);
}

// D: head_dim, NH: KV heads (all in one tile), RK: rows kept per head (8 or 16 >= group),
// MAXB: sequences the shared-memory tables hold.
template <int D, int NH, int RK, int MAXB> struct DecodeShape {
  static constexpr int TILE = kBS * D * 2;             // one head's K (or V) of one block
  static constexpr int STAGE = NH * TILE;              // K (or V) of all heads of one block
  static constexpr int WPH = kNC / NH;                 // consumer warps per KV head
  static constexpr int DP = D + 4;                     // padded combine row (no bank conflicts)
  static constexpr int WARP_STATE = 2 * RK + RK * DP;  // floats: m[RK], l[RK], O[RK][DP]
  static constexpr int TABLES = 4 * (MAXB + 1) * 4;  // lengths, table rows, two prefix sums
  // A head's warps merge their states at the end of a segment either all at once (every
  // warp's state in shared memory, all warps combining) or pairwise (half of them hand
  // their state to the other half, down to one: WPH / 2 states per head). Pairwise takes
  // more barriers and is used only where its smaller buffer deepens a two-per-SM ring.
  static constexpr int COMB_ALL = kNC * WARP_STATE * 4;
  static constexpr int COMB_PAIR = NH * (WPH / 2) * WARP_STATE * 4;
  static constexpr bool PAIR =
      ring_two(1024 + COMB_PAIR + TABLES + 256, STAGE, WPH, RK) &&
      ring_two(1024 + COMB_ALL + TABLES + 256, STAGE, WPH, RK) &&
      ring_pw(1024 + COMB_PAIR + TABLES + 256, STAGE, WPH, RK) > ring_pw(1024 + COMB_ALL + TABLES + 256, STAGE, WPH, RK);
  static constexpr int COMB = PAIR ? COMB_PAIR : COMB_ALL;
  static constexpr int FIXED = 1024 + COMB + TABLES + 256;
  static constexpr bool TWO = ring_two(FIXED, STAGE, WPH, RK);
  static constexpr int PW = ring_pw(FIXED, STAGE, WPH, RK);
  static constexpr int S = WPH * PW;
  static constexpr int RING = 2 * S * STAGE;
  static constexpr int SMEM = 1024 + RING + COMB + TABLES + 2 * S * 8;
  static constexpr int MIN_BLOCKS = TWO ? 2 : 1;
  static_assert(PW >= 1, "ring too shallow");
};

struct DecodeParams {
  void* out;
  const void* q;
  const void* k_new;
  const void* v_new;
  void* k_pool;
  void* v_pool;
  const int64_t* slot_mapping;
  const int32_t* tables;
  const int32_t* seq_rows;
  const int32_t* context_lens;
  int32_t* status;
  int32_t* counters;  // [kMaxBatch] segments of each sequence finished so far
  float* partials;    // [max_slots][NH][RK][D + 4]: (m, l, pad, pad, O) per row of a segment
  int64_t out_sb, out_sh, q_sb, q_sh, kv_sb, kv_sh, table_stride;
  int32_t table_rows, table_cols;
  int32_t batch, group, kv_heads, layer, nbt, inputs_ready, max_slots, cap_override;
  int32_t flat_min, min_quota;
  float scale_log2;
  // RoPE fused in (pkv_decode_attention_rope): q and the new k are the raw qkv_proj rows,
  // rotated here at position context_lens[b] - 1 with these [max_positions, D] tables.
  const void* rope_cos;
  const void* rope_sin;
  int64_t rope_max_pos;
};

__device__ inline void named_bar(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ inline int warp_sum(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Inclusive scan over the warp.
__device__ inline int warp_scan(int v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += u;
  }
  return v;
}

// Largest b in [lo, hi] with cum[b] <= k.
__device__ inline int seq_of(const int* cum, int k, int lo, int hi) {
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cum[mid] <= k) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// One run of consecutive blocks [i0, i1) of sequence b. A cut one (parts > 1) is part
// `part` of its sequence and keeps its partial state in `slot`.
struct Seg {
  int b, i0, i1, part, parts, slot;
};

// The CTA's segments in order, under either split (see the top of this file). sA holds
// per-sequence prefix sums: of blocks (equal ranges) or of units (chunks); sB the prefix
// sums of cut units (chunks only).
template <bool FLAT_OK>
struct SegIter {
  const int* sA;
  const int* sB;
  const int* sCtx;
  int B, C, g, flat, q, k0, k1, cur;  // cur: the last unit (chunks) or sequence (ranges) handed out
  __device__ int blocks(int b) const { return (sCtx[b] + kBS - 1) / kBS; }
  __device__ void start() {
    if (FLAT_OK && flat) cur = k1 > k0 ? seq_of(sA, k0, 0, B - 1) - 1 : B;  // the sequence holding block k0, minus one
    else cur = g - C;
  }
  __device__ bool next(Seg& s) {
    if (FLAT_OK && flat) {
      int b = cur + 1;
      for (; b < B; ++b) {
        if (sA[b] >= k1) return false;
        if (sA[b + 1] > sA[b]) break;
      }
      if (b >= B) return false;
      cur = b;
      const int first = sA[b], last = sA[b + 1];
      s.b = b;
      s.i0 = max(first, k0) - first;
      s.i1 = min(last, k1) - first;
      const int f = first / q;
      s.parts = (last - 1) / q - f + 1;
      s.part = g - f;
      // A CTA keeps its first segment's state (a sequence that starts at or before k0) in
      // slot 2g and its last one's in 2g + 1; slot_of() reads them back by the same rule.
      s.slot = 2 * g + (first <= k0 ? 0 : 1);
      return true;
    }
    const int u = cur + C;
    if (u >= sA[B]) return false;
    cur = u;
    const int b = seq_of(sA, u, 0, B - 1);  // the (non-empty) sequence owning unit u
    const int nch = sA[b + 1] - sA[b], c = u - sA[b], n = blocks(b);
    const int cs = (n + nch - 1) / nch;
    s.b = b;
    s.i0 = c * cs;
    s.i1 = min(n, s.i0 + cs);
    s.parts = nch;
    s.part = c;
    s.slot = sB[b] + c;
    return true;
  }
  // Slot of part c of sequence b (for the merge).
  __device__ int slot_of(int b, int c) const {
    if (!FLAT_OK || !flat) return sB[b] + c;
    const int first = sA[b], f = first / q;
    return c == 0 ? 2 * f + (first == f * q ? 0 : 1) : 2 * (f + c);
  }
};

template <typename T, int D>
__device__ inline void load_q(uint32_t (&qa)[D / 16][4], const T* qb, int64_t q_sh, int G, int g_lane, int t4) {
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const int c0 = kk * 16 + 2 * t4;
    qa[kk][0] = g_lane < G ? *reinterpret_cast<const uint32_t*>(qb + g_lane * q_sh + c0) : 0u;
    qa[kk][1] = g_lane + 8 < G ? *reinterpret_cast<const uint32_t*>(qb + (g_lane + 8) * q_sh + c0) : 0u;
    qa[kk][2] = g_lane < G ? *reinterpret_cast<const uint32_t*>(qb + g_lane * q_sh + c0 + 8) : 0u;
    qa[kk][3] = g_lane + 8 < G ? *reinterpret_cast<const uint32_t*>(qb + (g_lane + 8) * q_sh + c0 + 8) : 0u;
  }
}

// FLAT_OK: the launch may take equal ranges (the host's bound on the batch's blocks
// reaches the threshold); without it the chunk rule is compiled alone.
// r(r(x * c) + r(y * s)) for a packed pair, each product and the sum in float32 and each
// rounded to T: the reference's apply_rope (engine/model.py:214-224) on eager fp16 / bf16
// tensors, so the rotated values are bit-identical to it on the same tables.
template <typename T>
__device__ inline uint32_t rope_pair(uint32_t x, uint32_t c, uint32_t y, uint32_t s) {
  const float2 xf = Dt<T>::unpack(x), cf = Dt<T>::unpack(c), yf = Dt<T>::unpack(y), sf = Dt<T>::unpack(s);
  const float2 a = Dt<T>::unpack(Dt<T>::pack(xf.x * cf.x, xf.y * cf.y));
  const float2 b = Dt<T>::unpack(Dt<T>::pack(yf.x * sf.x, yf.y * sf.y));
  return Dt<T>::pack(a.x + b.x, a.y + b.y);
}

// -x of both halves (exact).
__device__ inline uint32_t neg_pair(uint32_t x) { return x ^ 0x80008000u; }

// Rotate the Q fragments (qa[kk][i]: columns kk * 16 + 2 t4 + {0, 1} (+ 8 for i >= 2)) at
// the cos / sin rows of one position: column c < D / 2 pairs with -x[c + D / 2], column
// c + D / 2 with x[c]; a thread holds both (fragments kk and kk + D / 32).
template <typename T, int D>
__device__ inline void rope_q(uint32_t (&qa)[D / 16][4], const T* crow, const T* srow, int t4) {
#pragma unroll
  for (int kk = 0; kk < D / 32; ++kk) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = kk * 16 + 2 * t4 + (i >= 2 ? 8 : 0), c2 = c + D / 2;
      const uint32_t x1 = qa[kk][i], x2 = qa[kk + D / 32][i];
      const uint32_t c1 = *reinterpret_cast<const uint32_t*>(crow + c), s1 = *reinterpret_cast<const uint32_t*>(srow + c);
      const uint32_t cc2 = *reinterpret_cast<const uint32_t*>(crow + c2), s2 = *reinterpret_cast<const uint32_t*>(srow + c2);
      qa[kk][i] = rope_pair<T>(x1, c1, neg_pair(x2), s1);
      qa[kk + D / 32][i] = rope_pair<T>(x2, cc2, x1, s2);
    }
  }
}

// CAPS: the instance for batches of more than C / 2 sequences, which tries the candidate
// chunk caps; the others keep the fallback rule alone (a prologue as short as it can be).
template <typename T, int D, int NH, int RK, int MAXB, bool FLAT_OK, bool CAPS>
__global__ void __launch_bounds__(kThreads, DecodeShape<D, NH, RK, MAXB>::MIN_BLOCKS)
    decode_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                  const DecodeParams p) {
  using S = DecodeShape<D, NH, RK, MAXB>;
  constexpr int TILE = S::TILE, STAGE = S::STAGE, NS = S::S, WPH = S::WPH, DP = S::DP, WS = S::WARP_STATE;
  constexpr int LANES = kIssueLanes < NS ? kIssueLanes : NS;  // the copies of one issue use distinct stages
  constexpr int ROW = D + 4;            // partial row: m, l, 2 pad floats, O[D] (O 16-byte aligned)
  constexpr int SLOT = NH * RK * ROW;   // floats of one segment's partial state (all heads)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring_k = smem;
  uint8_t* ring_v = smem + NS * STAGE;
  float* comb = reinterpret_cast<float*>(smem + S::RING);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::RING + S::COMB);
  uint64_t* empty = full + NS;
  int* sCtx = reinterpret_cast<int*>(empty + NS);  // [batch] clamped context lengths
  int* sRow = sCtx + MAXB + 1;                     // [batch] block-table row of each sequence
  int* sA = sRow + MAXB + 1;                       // [batch + 1] blocks (ranges) or units (chunks) before b
  int* sB = sA + MAXB + 1;                         // [batch + 1] cut units before b (chunks)
  __shared__ int s_bad, s_npend, s_flat, s_q, s_total;
  __shared__ int2 s_pend[kMaxPending];  // (sequence, parts) of cut segments
  __shared__ int s_last[kMaxPending];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g_lane = lane >> 2, t4 = lane & 3;
  const int B = p.batch, G = p.group;
  const int C = gridDim.x, g = blockIdx.x;
  const int cap_tokens = p.table_cols * kBS;

  // With programmatic dependent launch this CTA may start while the previous kernel in
  // the stream drains; let the next kernel launch early too. Everything the previous
  // kernel may have produced is read only after grid_dep_wait(). With inputs_ready the
  // caller guarantees that context lengths, table rows and the cached K/V were complete
  // before the previous kernel began, so the prologue, the block lookups and the first
  // ring fill run before the wait, overlapping the previous kernel's tail; q, the new
  // rows, the append, the output and the workspace still come after it.
  grid_dep_launch_dependents();
  if (!p.inputs_ready) grid_dep_wait();

  // The split's per-sequence sums in three barrier-separated passes over chunks of 32
  // sequences, chunk c held by warp c % 9 (one chunk per warp up to 288 sequences):
  // (1) load lengths and table rows, chunk sums of blocks and non-empty sequences, and the
  //     units each candidate cap would make (lane k of a warp keeps candidate k's count);
  // (2) the rule and the cap from the totals, chunk-local scans of units / blocks;
  // (3) add the chunks' carries. Each warp works on its own chunks in parallel.
  __shared__ int s_ct[32], s_ci[32], s_ca[32], s_cb[32];
  __shared__ int s_cand[CAPS ? kNC + 1 : 1][kNumCaps];
  const int nchunks = (B + 31) / 32;
  int cand = 0;
  for (int base = warp * 32; base < B; base += kThreads) {
    const int i = base + lane;
    int n = 0;
    if (i < B) {
      int ctx = p.context_lens[i];
      int row = p.seq_rows ? p.seq_rows[i] : i;
      if (ctx > cap_tokens) {
        report(p.status, PKV_ERR_OUT_OF_RANGE);
        ctx = cap_tokens;
      }
      if (row >= p.table_rows) {
        report(p.status, PKV_ERR_OUT_OF_RANGE);
        row = -1;
      }
      ctx = max(ctx, 0);
      sCtx[i] = ctx;
      sRow[i] = row;
      n = (ctx + kBS - 1) / kBS;
    }
    const int ct = warp_sum(n), ci = warp_sum(n > 0);
    if (lane == 0) {
      s_ct[base / 32] = ct;
      s_ci[base / 32] = ci;
    }
    if constexpr (CAPS) {
#pragma unroll
      for (int k = 0; k < kNumCaps; ++k) {
        const int u = __reduce_add_sync(0xffffffffu, (n + cap_candidate(k) - 1) / cap_candidate(k));
        if (lane == k) cand += u;
      }
    }
  }
  if constexpr (CAPS) {
    if (lane < kNumCaps) s_cand[warp][lane] = cand;
  }
  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NH);  // one consumer warp per head releases each stage
    }
    fence_mbar_init();
    s_bad = 0;
    s_npend = 0;
  }
  __syncthreads();
  {
    const int tiles = warp_sum(lane < nchunks ? s_ct[lane] : 0);
    const int items = warp_sum(lane < nchunks ? s_ci[lane] : 0);
    const int flat = FLAT_OK && p.cap_override <= 0 && tiles >= p.flat_min * C;
    const int free_ctas = max(C - items, max(C / 4, 1));
    int cap = p.cap_override > 0 ? p.cap_override : max(kMinCap, (tiles + free_ctas - 1) / free_ctas);
    if constexpr (CAPS) {
      int units = 0, my_cap = 0;
#pragma unroll
      for (int k = 0; k < kNumCaps; ++k) my_cap = lane == k ? cap_candidate(k) : my_cap;
      if (lane < kNumCaps) {
#pragma unroll
        for (int w = 0; w <= kNC; ++w) units += s_cand[w][lane];
      }
      const unsigned fits = __ballot_sync(0xffffffffu, lane < kNumCaps && units <= C * 29 / 32);
      if (p.cap_override <= 0 && fits) cap = __shfl_sync(0xffffffffu, my_cap, __ffs(fits) - 1);
    }
    for (int base = warp * 32; base < B; base += kThreads) {
      const int i = base + lane;
      const int n = i < B ? (sCtx[i] + kBS - 1) / kBS : 0;
      const int nch = n == 0 ? 0 : (n <= cap ? 1 : (n + cap - 1) / cap);
      const int pa = warp_scan(flat ? n : nch, lane), pb = warp_scan(nch > 1 ? nch : 0, lane);
      if (i < B) {
        sA[i + 1] = pa;
        sB[i + 1] = pb;
      }
      if (lane == 31) {
        s_ca[base / 32] = pa;
        s_cb[base / 32] = pb;
      }
    }
    if (tid == 0) {
      s_flat = flat;
      s_q = max(p.min_quota, (tiles + C - 1) / C);
    }
  }
  __syncthreads();
  {
    const int va = lane < nchunks ? s_ca[lane] : 0, vb = lane < nchunks ? s_cb[lane] : 0;
    const int ia = warp_scan(va, lane), ib = warp_scan(vb, lane);
    const int ea = ia - va, eb = ib - vb;  // units / blocks before chunk `lane`
    for (int base = warp * 32; base < B; base += kThreads) {
      const int i = base + lane;
      const int ca = __shfl_sync(0xffffffffu, ea, base / 32), cb = __shfl_sync(0xffffffffu, eb, base / 32);
      if (i < B) {
        sA[i + 1] += ca;
        sB[i + 1] += cb;
      }
    }
    const int total = __shfl_sync(0xffffffffu, ia, 31);
    if (tid == 0) {
      sA[0] = sB[0] = 0;
      s_total = total;
    }
  }
  __syncthreads();
  const int flat = s_flat, q = s_q;
  // Cut units never exceed 2 * C (a candidate cap keeps all units within 29 / 32 of the
  // CTAs, the fallback rule cut units within 2 * max(C - I, C / 4)) and cut ranges 2 * C,
  // the slots the host provides (an overriding cap may ask for more).
  if (!flat && sB[B] > p.max_slots) {
    if (tid == 0) report(p.status, PKV_ERR_WORKSPACE);
    return;
  }
  SegIter<FLAT_OK> segs{sA, sB, sCtx, B, C, g, flat, q, 0, 0, 0};
  if (flat) {
    segs.k0 = min(s_total, g * q);
    segs.k1 = min(s_total, segs.k0 + q);
  }

  if (warp == kNC) {
    // ---------------------------------------------------------------- producer
    Seg sg;
    const uint64_t pol = policy_evict_first();
    bool ok = true, waited = false;
    uint64_t deadline = 0;
    int j = 0;  // blocks of this CTA issued so far
    segs.start();
    while (ok && segs.next(sg)) {
      const int row = sRow[sg.b];
      auto lookup = [&](int i) -> int {  // block id of block i of the segment's sequence
        if (i >= sg.i1) return 0;
        int blk = row >= 0 ? p.tables[row * p.table_stride + i] : p.nbt - 1;  // padding rows: scratch block
        if (blk < 0 || blk >= p.nbt) {
          report(p.status, PKV_ERR_OUT_OF_RANGE);
          blk = p.nbt - 1;
        }
        return blk;
      };
      int blk_next = lookup(sg.i0 + lane);
      for (int base = sg.i0; base < sg.i1 && ok; base += 32) {
        const int blk_cur = blk_next;
        blk_next = lookup(base + 32 + lane);  // in flight while this batch is issued
        const int cnt = min(32, sg.i1 - base);
        for (int k0 = 0; k0 < cnt && ok; k0 += LANES) {
          const int blk = __shfl_sync(0xffffffffu, blk_cur, (k0 + lane) & 31);
          if (!waited && j + k0 + LANES > NS) {
            // Stages are reused from here on; their consumers start after the previous
            // kernel, and the wait budget starts with them.
            grid_dep_wait();
            waited = true;
            deadline = global_ns() + kWaitBudgetNs;
          }
          bool lok = true;
          if (lane < LANES && k0 + lane < cnt) {
            const int jj = j + k0 + lane, st = jj % NS;
            if (jj >= NS && !mbar_wait_until(&empty[st], ((jj / NS) - 1) & 1, deadline)) {
              report(p.status, PKV_ERR_TIMEOUT);
              lok = false;
            }
            if (lok) {
              const int c4 = p.layer * p.nbt + blk;
              mbar_arrive_expect_tx(&full[st], 2 * STAGE);
              tma_load_5d(ring_k + st * STAGE, &tmap_k, 0, 0, 0, 0, c4, &full[st], pol);
              tma_load_5d(ring_v + st * STAGE, &tmap_v, 0, 0, 0, 0, c4, &full[st], pol);
            }
          }
          ok = __all_sync(0xffffffffu, lok);
        }
        j += cnt;
      }
    }
    if (!waited) grid_dep_wait();
    if (!ok) s_bad = 1;
  } else {
    // ---------------------------------------------------------------- consumers
    grid_dep_wait();  // q, the new rows, the output and the pool writes depend on earlier kernels
    const uint64_t deadline = global_ns() + kWaitBudgetNs;
    if (g == C - 1) {  // sequences with nothing to attend to get zeros (the reference never asks for this)
      for (int b = warp; b < B; b += kNC) {
        if (sCtx[b] != 0) continue;
        T* o = reinterpret_cast<T*>(p.out) + b * p.out_sb;
        for (int e = lane; e < NH * G * D; e += 32) o[(e / D) * p.out_sh + e % D] = Dt<T>::from_f(0.f);
      }
    }
    const int h = warp / WPH, w = warp % WPH;  // this warp's KV head and its rank among the head's warps
    float* head_comb = comb + h * (S::PAIR ? WPH / 2 : WPH) * WS;  // this head's merge states
    bool ok = true;
    int j = 0;  // blocks of this CTA consumed so far (by all warps)
    Seg sg;
    segs.start();
    while (segs.next(sg)) {
      // Q fragments of this head's query group (A operand, rows = query heads).
      uint32_t qa[D / 16][4];
      load_q<T, D>(qa, reinterpret_cast<const T*>(p.q) + sg.b * p.q_sb + (int64_t)h * G * p.q_sh, p.q_sh, G, g_lane,
                   t4);
      const T* rope_c = nullptr;
      const T* rope_s = nullptr;
      if (p.rope_cos) {  // rows at the new token's position (rows >= G are zero and stay zero)
        int64_t pos = sCtx[sg.b] - 1;
        if (pos >= p.rope_max_pos) {
          if (lane == 0) report(p.status, PKV_ERR_OUT_OF_RANGE);
          pos = 0;
        }
        rope_c = reinterpret_cast<const T*>(p.rope_cos) + pos * D;
        rope_s = reinterpret_cast<const T*>(p.rope_sin) + pos * D;
        rope_q<T, D>(qa, rope_c, rope_s, t4);
      }
      const int b = sg.b;
      const int ctx = sCtx[b];
      const int append_blk = p.k_new ? (ctx - 1) / kBS : -1;
      float m_r[2] = {-INFINITY, -INFINITY};
      float l_r[2] = {0.f, 0.f};
      float o[D / 8][4];
#pragma unroll
      for (int jj = 0; jj < D / 8; ++jj) o[jj][0] = o[jj][1] = o[jj][2] = o[jj][3] = 0.f;

      const int n_i = sg.i1 - sg.i0;
      for (int k = ((w - j) % WPH + WPH) % WPH; k < n_i; k += WPH) {
        const int jj = j + k, st = jj % NS;
        if (ok && !mbar_wait_until(&full[st], (jj / NS) & 1, deadline)) {
          report(p.status, PKV_ERR_TIMEOUT);
          ok = false;
        }
        if (ok) {
          uint8_t* kt = ring_k + st * STAGE + h * TILE;
          uint8_t* vt = ring_v + st * STAGE + h * TILE;
          const int i = sg.i0 + k;  // block index within the sequence
          if (i == append_blk) {
            // Put the new row into the staged tiles and write it to the pool at slot_mapping[b].
            const int off = (ctx - 1) % kBS;
            const int64_t slot = p.slot_mapping[b];
            const bool write = slot >= 0 && slot < (int64_t)p.nbt * kBS;
            if (slot >= (int64_t)p.nbt * kBS && lane == 0) report(p.status, PKV_ERR_OUT_OF_RANGE);
            const T* kn = reinterpret_cast<const T*>(p.k_new) + b * p.kv_sb + h * p.kv_sh;
            const T* vn = reinterpret_cast<const T*>(p.v_new) + b * p.kv_sb + h * p.kv_sh;
            const int64_t dst =
                (((int64_t)p.layer * p.nbt + (write ? slot / kBS : 0)) * NH + h) * kBS * D + (write ? slot % kBS : 0) * D;
#pragma unroll
            for (int wd = lane; wd < D / 2; wd += 32) {
              const int d0 = 2 * wd;
              uint32_t kw = *reinterpret_cast<const uint32_t*>(kn + d0);
              const uint32_t vw = *reinterpret_cast<const uint32_t*>(vn + d0);
              if (rope_c) {  // the new key rotated as q: its partner is D / 2 away
                const uint32_t kp = *reinterpret_cast<const uint32_t*>(kn + (d0 ^ (D / 2)));
                kw = rope_pair<T>(kw, *reinterpret_cast<const uint32_t*>(rope_c + d0), d0 < D / 2 ? neg_pair(kp) : kp,
                                  *reinterpret_cast<const uint32_t*>(rope_s + d0));
              }
              const uint32_t r = (d0 / 64) * kBS + off;
              *reinterpret_cast<uint32_t*>(kt + swz128(r, d0 % 64)) = kw;
              *reinterpret_cast<uint32_t*>(vt + swz128(r, d0 % 64)) = vw;
              if (write) {
                *reinterpret_cast<uint32_t*>(reinterpret_cast<T*>(p.k_pool) + dst + d0) = kw;
                *reinterpret_cast<uint32_t*>(reinterpret_cast<T*>(p.v_pool) + dst + d0) = vw;
              }
            }
            __syncwarp();
          }
          attend_tile16<T, D>(qa, smem_u32(kt), smem_u32(vt), i * kBS, [ctx](int, int key) { return key < ctx; },
                              p.scale_log2, m_r, l_r, o);
        }
        // This warp's generic accesses to the stage come before the producer's next
        // async-proxy fill of it.
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
      }
      finish_row_sums(l_r);
      const bool whole = sg.parts == 1;
      float* part = p.partials + (int64_t)sg.slot * SLOT + h * RK * ROW;
      T* outp = reinterpret_cast<T*>(p.out) + b * p.out_sb + (int64_t)h * G * p.out_sh;
      if constexpr (S::PAIR) {
        // Merge the head's warps pairwise: in each round the upper half of the remaining
        // warps hands its state (m, l and O of rows g_lane, g_lane + 8 in the MMA fragment
        // layout) through a slot to the lower half, which folds it into its registers. Warp 0
        // of the head ends with the segment's state.
#pragma unroll
        for (int half = WPH / 2; half >= 1; half >>= 1) {
          if (w >= half && w < 2 * half) {
            float* c = head_comb + (w - half) * WS;
            if (t4 == 0) {
              c[g_lane] = m_r[0];
              c[RK + g_lane] = l_r[0];
              if (RK > 8) {
                c[g_lane + 8] = m_r[1];
                c[RK + g_lane + 8] = l_r[1];
              }
            }
#pragma unroll
            for (int jj = 0; jj < D / 8; ++jj) {
              const int col = 8 * jj + 2 * t4;
              *reinterpret_cast<float2*>(&c[2 * RK + g_lane * DP + col]) = make_float2(o[jj][0], o[jj][1]);
              if (RK > 8) *reinterpret_cast<float2*>(&c[2 * RK + (g_lane + 8) * DP + col]) = make_float2(o[jj][2], o[jj][3]);
            }
          }
          named_bar(1 + h, WPH * 32);
          if (w < half) {
            const float* c = head_comb + w * WS;
            float fa[2], fb[2];
#pragma unroll
            for (int i = 0; i < (RK > 8 ? 2 : 1); ++i) {
              const float mb = c[g_lane + 8 * i], lb = c[RK + g_lane + 8 * i];
              const float mn = fmaxf(m_r[i], mb);
              const float mref = mn == -INFINITY ? 0.f : mn;  // both empty: weights 0, not NaN
              fa[i] = ex2(m_r[i] - mref);
              fb[i] = ex2(mb - mref);
              m_r[i] = mn;
              l_r[i] = l_r[i] * fa[i] + lb * fb[i];
            }
#pragma unroll
            for (int jj = 0; jj < D / 8; ++jj) {
              const int col = 8 * jj + 2 * t4;
              const float2 v = *reinterpret_cast<const float2*>(&c[2 * RK + g_lane * DP + col]);
              o[jj][0] = o[jj][0] * fa[0] + v.x * fb[0];
              o[jj][1] = o[jj][1] * fa[0] + v.y * fb[0];
              if (RK > 8) {
                const float2 u = *reinterpret_cast<const float2*>(&c[2 * RK + (g_lane + 8) * DP + col]);
                o[jj][2] = o[jj][2] * fa[1] + u.x * fb[1];
                o[jj][3] = o[jj][3] * fa[1] + u.y * fb[1];
              }
            }
          }
          named_bar(1 + h, WPH * 32);  // the slots are written again by the next round or segment
        }
        if (w == 0) {
#pragma unroll
          for (int i = 0; i < (RK > 8 ? 2 : 1); ++i) {
            const int r = g_lane + 8 * i;
            if (r >= G) continue;
            if (whole) {
              const float inv = 1.f / l_r[i];
#pragma unroll
              for (int jj = 0; jj < D / 8; ++jj)
                *reinterpret_cast<uint32_t*>(outp + r * p.out_sh + 8 * jj + 2 * t4) =
                    Dt<T>::pack(o[jj][2 * i] * inv, o[jj][2 * i + 1] * inv);
            } else {
#pragma unroll
              for (int jj = 0; jj < D / 8; ++jj)
                __stcg(reinterpret_cast<float2*>(part + r * ROW + 4 + 8 * jj + 2 * t4),
                       make_float2(o[jj][2 * i], o[jj][2 * i + 1]));
              if (t4 == 0) __stcg(reinterpret_cast<float2*>(part + r * ROW), make_float2(m_r[i], l_r[i]));
            }
          }
        }
      } else {
        // Every warp of the head puts its state in shared memory; all of them then combine
        // the states column by column.
        float* cm = head_comb + w * WS;
        float* cl = cm + RK;
        float* co = cl + RK;
        if (t4 == 0) {
          cm[g_lane] = m_r[0];
          cl[g_lane] = l_r[0];
          if (RK > 8) {
            cm[g_lane + 8] = m_r[1];
            cl[g_lane + 8] = l_r[1];
          }
        }
#pragma unroll
        for (int jj = 0; jj < D / 8; ++jj) {
          const int col = 8 * jj + 2 * t4;
          *reinterpret_cast<float2*>(&co[g_lane * DP + col]) = make_float2(o[jj][0], o[jj][1]);
          if (RK > 8) *reinterpret_cast<float2*>(&co[(g_lane + 8) * DP + col]) = make_float2(o[jj][2], o[jj][3]);
        }
        named_bar(1 + h, WPH * 32);
        for (int it = w * 32 + lane; it < G * (D / 2); it += WPH * 32) {
          const int r = it / (D / 2), col = 2 * (it % (D / 2));
          float mm = -INFINITY;
#pragma unroll
          for (int ww = 0; ww < WPH; ++ww) mm = fmaxf(mm, head_comb[ww * WS + r]);
          float ll = 0.f, o0 = 0.f, o1 = 0.f;
#pragma unroll
          for (int ww = 0; ww < WPH; ++ww) {
            const float* c = head_comb + ww * WS;
            const float f = ex2(c[r] - mm);  // a warp without tiles has m = -inf: f = 0
            ll += c[RK + r] * f;
            const float2 v = *reinterpret_cast<const float2*>(&c[2 * RK + r * DP + col]);
            o0 += v.x * f;
            o1 += v.y * f;
          }
          if (whole) {
            const float inv = 1.f / ll;
            *reinterpret_cast<uint32_t*>(outp + r * p.out_sh + col) = Dt<T>::pack(o0 * inv, o1 * inv);
          } else {
            __stcg(reinterpret_cast<float2*>(part + r * ROW + 4 + col), make_float2(o0, o1));
            if (col == 0) __stcg(reinterpret_cast<float2*>(part + r * ROW), make_float2(mm, ll));
          }
        }
        named_bar(1 + h, WPH * 32);  // the states are written again by the next segment
      }
      if (!whole && warp == 0 && lane == 0) {
        // The launcher refuses launches where a CTA could hold more cut segments than this.
        if (s_npend < kMaxPending) s_pend[s_npend++] = make_int2(b, sg.parts);
        else report(p.status, PKV_ERR_WORKSPACE);
      }
      j += n_i;
    }
    if (!ok) s_bad = 1;
  }
  __syncthreads();
  const int npend = s_npend;
  if (npend == 0) return;

  // Tickets for this CTA's cut segments; the CTA holding the last ticket of a sequence
  // merges it. The barrier orders every consumer's partial writes before thread 0's
  // tickets, whose release publishes them; for the last holder the same atomic's acquire
  // (then the barrier below) orders the other segments' partials before its threads'
  // reads. One acquire-release atomic per ticket measured faster than fence + atomic + fence.
  if (tid == 0) {
    for (int k0 = 0; k0 < npend; k0 += kTicketBatch) {
      int ticket[kTicketBatch];
#pragma unroll
      for (int k = 0; k < kTicketBatch; ++k)  // a batch in flight together
        if (k0 + k < npend) ticket[k] = atom_add_acq_rel_gpu(p.counters + s_pend[k0 + k].x, 1);
#pragma unroll
      for (int k = 0; k < kTicketBatch; ++k) {
        if (k0 + k >= npend) break;
        const bool last = ticket[k] == s_pend[k0 + k].y - 1;
        if (last) p.counters[s_pend[k0 + k].x] = 0;  // ready for the next call
        s_last[k0 + k] = last;
      }
    }
  }
  __syncthreads();
  if (warp == kNC || s_bad) return;
  for (int k = 0; k < npend; ++k) {
    if (!s_last[k]) continue;
    const int b = s_pend[k].x, parts = s_pend[k].y;
    for (int it = tid; it < NH * G * (D / 4); it += kNC * 32) {
      const int c = (it % (D / 4)) * 4;
      const int hr = it / (D / 4), h = hr / G, r = hr - h * G;
      float mx = -INFINITY, l = 0.f, a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      for (int q0 = 0; q0 < parts; q0 += kMergeBatch) {
        const int cnt = min(kMergeBatch, parts - q0);
        float2 ml[kMergeBatch];
        float4 ov[kMergeBatch];
#pragma unroll
        for (int x = 0; x < kMergeBatch; ++x) {
          if (x < cnt) {
            const float* row = p.partials + (int64_t)segs.slot_of(b, q0 + x) * SLOT + (h * RK + r) * ROW;
            ml[x] = __ldcg(reinterpret_cast<const float2*>(row));
            ov[x] = __ldcg(reinterpret_cast<const float4*>(row + 4 + c));
          }
        }
        float mn = mx;
#pragma unroll
        for (int x = 0; x < kMergeBatch; ++x)
          if (x < cnt) mn = fmaxf(mn, ml[x].x);
        const float fo = mx == -INFINITY ? 0.f : ex2(mx - mn);
        l *= fo, a0 *= fo, a1 *= fo, a2 *= fo, a3 *= fo;
#pragma unroll
        for (int x = 0; x < kMergeBatch; ++x) {
          if (x < cnt) {
            const float f = ex2(ml[x].x - mn);
            l += ml[x].y * f;
            a0 += ov[x].x * f, a1 += ov[x].y * f, a2 += ov[x].z * f, a3 += ov[x].w * f;
          }
        }
        mx = mn;
      }
      const float inv = 1.f / l;
      T* outp = reinterpret_cast<T*>(p.out) + b * p.out_sb + (int64_t)(h * G + r) * p.out_sh + c;
      *reinterpret_cast<uint32_t*>(outp) = Dt<T>::pack(a0 * inv, a1 * inv);
      *reinterpret_cast<uint32_t*>(outp + 2) = Dt<T>::pack(a2 * inv, a3 * inv);
    }
  }
}

// Workspace: [ticket counters: kMaxBatch int32][partials: 2 * ctas slots of
// NH * RK * (D + 4) floats]. The counters start at zero and every call leaves them at zero.
constexpr int kMaxCtas = 4 * 256;  // workspace is sized for up to 4 CTAs on each of up to 256 SMs
constexpr int64_t kPartialsOffset = (int64_t)kMaxBatch * 4;
int64_t ws_bytes(int ctas, int nh, int rk, int d) { return kPartialsOffset + (int64_t)2 * ctas * nh * rk * (d + 4) * 4; }

// Tuning knobs, read once from the environment (0 / unset = built-in choice):
//   PKV_DECODE_CTAS_PER_SM  CTAs per SM (at most what the shared memory allows)
//   PKV_DECODE_CTAS         CTAs in all (at most CTAs per SM x SMs)
//   PKV_DECODE_PDL          0 = launch without programmatic stream serialization
//   PKV_DECODE_CAP          chunks of at most this many blocks (no equal ranges)
//   PKV_DECODE_FLAT_MIN     blocks per CTA from which the ranges are equal
//   PKV_DECODE_SMALL_TABLES 0 = every batch takes the instance with tables for kMaxBatch
struct DecodeKnobs {
  int ctas_per_sm = 0, ctas = 0, pdl = 1, cap = 0, flat_min = 0, small_tables = 1;
  DecodeKnobs() {
    auto env = [](const char* k, int dflt) {
      const char* v = getenv(k);
      return v && *v ? atoi(v) : dflt;
    };
    ctas_per_sm = env("PKV_DECODE_CTAS_PER_SM", 0);
    ctas = env("PKV_DECODE_CTAS", 0);
    pdl = env("PKV_DECODE_PDL", 1);
    cap = env("PKV_DECODE_CAP", 0);
    flat_min = env("PKV_DECODE_FLAT_MIN", 0);
    small_tables = env("PKV_DECODE_SMALL_TABLES", 1);
  }
};
const DecodeKnobs& knobs() {
  static const DecodeKnobs k;
  return k;
}

template <typename T, int D, int NH, int RK, int MAXB, bool FLAT_OK, bool CAPS>
int launch_decode(const pkv_pool& pool, const DecodeParams& p0, void* workspace, int64_t workspace_bytes,
                  cudaStream_t stream) {
  using S = DecodeShape<D, NH, RK, MAXB>;
  if (p0.batch > MAXB) return PKV_ERR_UNSUPPORTED;
  static int per_sm = 0;
  if (per_sm == 0) {
    cudaError_t e =
        cudaFuncSetAttribute(decode_kernel<T, D, NH, RK, MAXB, FLAT_OK, CAPS>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM);
    if (e != cudaSuccess) return cuda_status(e);
    int occ = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, decode_kernel<T, D, NH, RK, MAXB, FLAT_OK, CAPS>, kThreads, S::SMEM);
    if (e != cudaSuccess) return cuda_status(e);
    per_sm = std::max(1, occ);
  }
  const int want = knobs().ctas_per_sm > 0 ? std::min(knobs().ctas_per_sm, per_sm) : per_sm;
  int ctas = std::min(num_sms() * want, kMaxCtas);
  if (knobs().ctas > 0) ctas = std::min(ctas, knobs().ctas);
  if (!workspace || workspace_bytes < ws_bytes(ctas, NH, RK, D)) return PKV_ERR_WORKSPACE;
  // With chunks a CTA holds at most ceil((batch + 2 * ctas) / ctas) units (whole sequences
  // plus the cut units' slots), so every cut unit's ticket fits its list (148+ SMs: always).
  if ((p0.batch + 2 * ctas + ctas - 1) / ctas > kMaxPending) return PKV_ERR_UNSUPPORTED;
  CUtensorMap tk, tv;
  if (!get_pool_maps(pool, &tk, &tv, NH)) return PKV_ERR_CUDA;
  DecodeParams p = p0;
  uint8_t* wsb = static_cast<uint8_t*>(workspace);
  p.counters = reinterpret_cast<int32_t*>(wsb);
  p.partials = reinterpret_cast<float*>(wsb + kPartialsOffset);
  p.max_slots = 2 * ctas;
  p.cap_override = knobs().cap;
  p.flat_min = knobs().flat_min > 0 ? knobs().flat_min : kFlatMin;
  p.min_quota = kMinQuota;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = S::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = knobs().pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, decode_kernel<T, D, NH, RK, MAXB, FLAT_OK, CAPS>, tk, tv, p));
}

template <typename T, int D, int NH, int RK, int MAXB>
int launch_split(const pkv_pool& pool, const DecodeParams& p, void* ws, int64_t wsb, cudaStream_t st) {
  // The batch attends to at most batch * table_cols blocks, and (unless sequences share
  // blocks) to no more than the pool holds: below the equal-range threshold for the CTAs
  // this shape launches, the chunk rule alone is compiled in. The bound only picks the
  // faster instance; the chunk rule is correct for any lengths.
  using S = DecodeShape<D, NH, RK, MAXB>;
  const int64_t bound = std::min<int64_t>((int64_t)p.batch * p.table_cols, pool.num_blocks_total);
  const int flat_min = knobs().flat_min > 0 ? knobs().flat_min : kFlatMin;
  const bool may_flat = knobs().cap <= 0 && bound >= (int64_t)flat_min * num_sms() * S::MIN_BLOCKS;
  if (may_flat) return launch_decode<T, D, NH, RK, MAXB, true, false>(pool, p, ws, wsb, st);
  // More sequences than half the CTAs this shape launches (two per SM at most): the
  // instance that tries the candidate chunk caps. Any instance is correct for any batch.
  if constexpr (MAXB == kSmallBatch) {
    if (knobs().cap <= 0 && (int64_t)p.batch * 2 > (int64_t)num_sms() * S::MIN_BLOCKS)
      return launch_decode<T, D, NH, RK, MAXB, false, true>(pool, p, ws, wsb, st);
  }
  return launch_decode<T, D, NH, RK, MAXB, false, false>(pool, p, ws, wsb, st);
}

// Batches of up to kSmallBatch sequences take the instance with small per-sequence tables,
// whose freed shared memory deepens the ring where the shape allows.
template <typename T, int D, int NH, int RK>
int launch_tables(const pkv_pool& pool, const DecodeParams& p, void* ws, int64_t wsb, cudaStream_t st) {
  return p.batch <= kSmallBatch && knobs().small_tables ? launch_split<T, D, NH, RK, kSmallBatch>(pool, p, ws, wsb, st)
                                : launch_split<T, D, NH, RK, kMaxBatch>(pool, p, ws, wsb, st);
}

template <typename T, int D, int NH>
int launch_rows(const pkv_pool& pool, const DecodeParams& p, void* ws, int64_t wsb, cudaStream_t st) {
  return p.group <= 8 ? launch_tables<T, D, NH, 8>(pool, p, ws, wsb, st)
                      : launch_tables<T, D, NH, 16>(pool, p, ws, wsb, st);
}

template <typename T, int D>
int launch_heads(const pkv_pool& pool, const DecodeParams& p, void* ws, int64_t wsb, cudaStream_t st) {
  switch (pool.num_kv_heads) {
    case 1: return launch_rows<T, D, 1>(pool, p, ws, wsb, st);
    case 2: return launch_rows<T, D, 2>(pool, p, ws, wsb, st);
    case 4: return launch_rows<T, D, 4>(pool, p, ws, wsb, st);
    case 8: return launch_rows<T, D, 8>(pool, p, ws, wsb, st);
    default: return PKV_ERR_UNSUPPORTED;
  }
}

}  // namespace
}  // namespace pkv

using namespace pkv;
using T16 = uint16_t;  // a 16-bit element of the pool's storage type

extern "C" int pkv_decode_reset_workspace(void* workspace, int64_t workspace_bytes, pkv_stream_t stream) {
  if (!workspace || workspace_bytes < kPartialsOffset) return PKV_ERR_INVALID_ARGUMENT;
  return cuda_status(cudaMemsetAsync(workspace, 0, kPartialsOffset, reinterpret_cast<cudaStream_t>(stream)));
}

extern "C" int64_t pkv_decode_workspace_bytes(int32_t batch, int32_t num_kv_heads, int32_t max_blocks_per_seq,
                                              int32_t block_size, int32_t head_dim, int32_t num_q_heads) {
  if (batch <= 0 || batch > kMaxBatch || max_blocks_per_seq <= 0 || block_size != kBS ||
      (head_dim != 64 && head_dim != 128) || num_q_heads <= 0)
    return 0;
  if (num_kv_heads != 1 && num_kv_heads != 2 && num_kv_heads != 4 && num_kv_heads != 8) return 0;
  if (num_q_heads % num_kv_heads != 0) return 0;
  const int group = num_q_heads / num_kv_heads;
  return ws_bytes(kMaxCtas, num_kv_heads, group <= 8 ? 8 : 16, head_dim);
}

namespace {

// Checks shared by the entry points and the launch; q, k_new, v_new and their strides are set.
int decode_launch(const pkv_pool* pool, int32_t layer, const pkv_tables* tables, int32_t batch, int32_t num_q_heads,
                  void* out, int64_t out_stride_b, int64_t out_stride_h, const int64_t* slot_mapping,
                  const int32_t* context_lens, float scale, int32_t flags, void* workspace, int64_t workspace_bytes,
                  int32_t* status_dev, pkv_stream_t stream, DecodeParams& p) {
  if (!pool || !tables || !out || !p.q || !context_lens || !tables->block_tables) return PKV_ERR_INVALID_ARGUMENT;
  if (batch < 0 || layer < 0 || layer >= pool->num_layers) return PKV_ERR_INVALID_ARGUMENT;
  if (batch == 0) return PKV_OK;
  if (batch > kMaxBatch) return PKV_ERR_UNSUPPORTED;
  const int d = pool->head_dim, hkv = pool->num_kv_heads;
  if (pool->block_size != kBS || (d != 64 && d != 128)) return PKV_ERR_UNSUPPORTED;
  if (hkv <= 0 || num_q_heads <= 0 || num_q_heads % hkv != 0) return PKV_ERR_INVALID_ARGUMENT;
  if (hkv != 1 && hkv != 2 && hkv != 4 && hkv != 8) return PKV_ERR_UNSUPPORTED;
  const int group = num_q_heads / hkv;
  if (group > 16) return PKV_ERR_UNSUPPORTED;
  if ((p.k_new == nullptr) != (p.v_new == nullptr)) return PKV_ERR_INVALID_ARGUMENT;
  if (p.k_new && !slot_mapping) return PKV_ERR_INVALID_ARGUMENT;
  // 32-bit accesses to q, out and the new rows: even strides, 4-byte aligned bases.
  auto aligned4 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 3) == 0; };
  if (!aligned4(p.q) || !aligned4(out) || (p.k_new && (!aligned4(p.k_new) || !aligned4(p.v_new))))
    return PKV_ERR_INVALID_ARGUMENT;
  if ((p.q_sb | p.q_sh | out_stride_b | out_stride_h) & 1) return PKV_ERR_INVALID_ARGUMENT;
  if (p.k_new && ((p.kv_sb | p.kv_sh) & 1)) return PKV_ERR_INVALID_ARGUMENT;
  if (tables->cols <= 0 || tables->rows <= 0) return PKV_ERR_INVALID_ARGUMENT;
  if (!tables->seq_rows && tables->rows < batch) return PKV_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return PKV_ERR_INVALID_ARGUMENT;

  p.out = out;
  p.k_pool = pool->k;
  p.v_pool = pool->v;
  p.slot_mapping = slot_mapping;
  p.tables = tables->block_tables;
  p.seq_rows = tables->seq_rows;
  p.context_lens = context_lens;
  p.status = status_dev;
  p.out_sb = out_stride_b;
  p.out_sh = out_stride_h;
  p.table_stride = tables->stride;
  p.table_rows = tables->rows;
  p.table_cols = tables->cols;
  p.batch = batch;
  p.group = group;
  p.kv_heads = hkv;
  p.layer = layer;
  p.nbt = pool->num_blocks_total;
  p.scale_log2 = scale * kLog2e;
  p.inputs_ready = (flags & PKV_DECODE_INPUTS_READY) ? 1 : 0;

  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (pool->dtype == PKV_F16) {
    return d == 64 ? launch_heads<__half, 64>(*pool, p, workspace, workspace_bytes, st)
                   : launch_heads<__half, 128>(*pool, p, workspace, workspace_bytes, st);
  }
  if (pool->dtype == PKV_BF16) {
    return d == 64 ? launch_heads<__nv_bfloat16, 64>(*pool, p, workspace, workspace_bytes, st)
                   : launch_heads<__nv_bfloat16, 128>(*pool, p, workspace, workspace_bytes, st);
  }
  return PKV_ERR_UNSUPPORTED;
}

}  // namespace

extern "C" int pkv_decode_attention(const pkv_pool* pool, int32_t layer, const pkv_tables* tables, int32_t batch,
                                    int32_t num_q_heads, void* out, int64_t out_stride_b, int64_t out_stride_h,
                                    const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k_new,
                                    const void* v_new, int64_t kv_stride_b, int64_t kv_stride_h,
                                    const int64_t* slot_mapping, const int32_t* context_lens, float scale,
                                    int32_t flags, void* workspace, int64_t workspace_bytes,
                                    int32_t* status_dev, pkv_stream_t stream) {
  DecodeParams p{};
  p.q = q;
  p.q_sb = q_stride_b;
  p.q_sh = q_stride_h;
  p.k_new = k_new;
  p.v_new = v_new;
  p.kv_sb = kv_stride_b;
  p.kv_sh = kv_stride_h;
  return decode_launch(pool, layer, tables, batch, num_q_heads, out, out_stride_b, out_stride_h, slot_mapping,
                       context_lens, scale, flags, workspace, workspace_bytes, status_dev, stream, p);
}

extern "C" int pkv_decode_attention_rope(const pkv_pool* pool, int32_t layer, const pkv_tables* tables, int32_t batch,
                                         int32_t num_q_heads, void* out, int64_t out_stride_b, int64_t out_stride_h,
                                         const void* qkv, int64_t qkv_stride, const void* cos_table,
                                         const void* sin_table, int64_t max_positions, const int64_t* slot_mapping,
                                         const int32_t* context_lens, float scale, int32_t flags, void* workspace,
                                         int64_t workspace_bytes, int32_t* status_dev, pkv_stream_t stream) {
  if (!pool || !qkv || !cos_table || !sin_table || !slot_mapping || max_positions <= 0) return PKV_ERR_INVALID_ARGUMENT;
  auto aligned4 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 3) == 0; };
  if (!aligned4(cos_table) || !aligned4(sin_table)) return PKV_ERR_INVALID_ARGUMENT;
  const int64_t d = pool->head_dim, hkv = pool->num_kv_heads;
  const T16* base = static_cast<const T16*>(qkv);
  DecodeParams p{};
  p.q = base;
  p.q_sb = qkv_stride;
  p.q_sh = d;
  p.k_new = base + num_q_heads * d;
  p.v_new = base + (num_q_heads + hkv) * d;
  p.kv_sb = qkv_stride;
  p.kv_sh = d;
  p.rope_cos = cos_table;
  p.rope_sin = sin_table;
  p.rope_max_pos = max_positions;
  return decode_launch(pool, layer, tables, batch, num_q_heads, out, out_stride_b, out_stride_h, slot_mapping,
                       context_lens, scale, flags, workspace, workspace_bytes, status_dev, stream, p);
}
