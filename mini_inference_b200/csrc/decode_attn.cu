// Paged decode attention for sm_100a, fused with the one-token KV append.
//
// Replaces, per layer and decode step, PagedDecodeContext.attend
// (engine/kv_cache.py:611-620): the index_put append, the gather of every
// sequence's blocks into a padded contiguous copy, and decode_attention's SDPA
// (engine/model.py:126-147). Here nothing is gathered: K/V blocks are read in
// place through the block table, each exactly once, straight into shared memory.
//
// Work split: one wave of CTAs that share the batch's blocks evenly. A "tile" is
// one block of one sequence with all its KV heads (K and V of all heads of a
// block are adjacent in the pool, so one 5-D TMA box per tensor fetches them).
// The batch's tiles, sequence after sequence, are cut into equal runs, one per
// CTA (every CTA computes the prefix sums of the per-sequence block counts from
// context_lens), so every CTA streams the same number of bytes whatever the mix
// of lengths.
//
// Inside a CTA one producer warp walks its run, resolves each tile's block id
// through the block table (32 at a time, one lookup per lane, the next 32
// already in flight) and keeps a ring of stages full with TMA copies (128B
// swizzle, L2 evict-first). 8 consumer warps split the KV heads (8 / Hkv warps
// per head) and take the run's tiles round-robin, each through stages of the
// ring that only it consumes, so that it waits on every phase of those stages'
// mbarriers in turn (a parity wait cannot tell a phase from the one two later).
// Each consumer runs the 16-key flash
// step on mma.sync m16n8k16 with the M = 16 rows being the GQA group's query
// heads (the reference regroups head h to (h / group, h % group) the same
// way), so a tile read from HBM serves the whole group (attn_tile.cuh), then
// hands the stage back to the producer through an mbarrier.
//
// A run covers pieces of consecutive sequences. At the end of a piece the warps
// of a head merge their softmax states through shared memory (a named barrier
// per head). A piece that is a whole sequence is written out directly; only the
// first and the last piece of a run can be partial, so a CTA keeps at most two
// partial states per head in the workspace. A second, small kernel launched right
// behind (programmatic dependent launch: it is resident early and waits on the
// decode grid) merges the pieces of each split sequence in run order; the CTA that
// holds a sequence's first piece leaves it a descriptor. No CTA waits on another
// and there are no atomics, so nothing in the workspace carries over between calls.
#include <algorithm>
#include <cstdlib>

#include "attn_tile.cuh"
#include "common.cuh"

namespace pkv {
namespace {

constexpr int kBS = 16;  // tokens per block handled by this kernel
constexpr int kNC = 8;   // consumer warps
constexpr int kThreads = (kNC + 1) * 32;
constexpr int kMaxBatch = 1024;  // the prefix sums live in shared memory
constexpr float kLog2e = 1.4426950408889634f;

// D: head_dim, NH: KV heads (all in one tile), RK: rows kept per head (8 or 16 >= group),
// DEEP: one CTA per SM with up to 6 ring stages per consumer warp.
template <int D, int NH, int RK, bool DEEP = false> struct DecodeShape {
  static constexpr int TILE = kBS * D * 2;  // one head's K (or V) for one block
  static constexpr int STAGE = NH * TILE;   // K (or V) of all heads of one block
  static constexpr int WPH = kNC / NH;      // consumer warps per KV head
  static constexpr int DP = D + 4;          // padded combine row (no bank conflicts)
  static constexpr int WARP_COMB = 2 * RK + RK * DP;        // floats: m[RK], l[RK], O[RK][DP]
  static constexpr int COMB = NH * WPH * WARP_COMB * 4;     // bytes
  static constexpr int PREFIX = 3 * (kMaxBatch + 1) * 4;    // block prefix sums, context lengths, table rows
  // Each consumer warp owns PW stages of the ring (see decode_kernel): S = WPH * PW.
  // Two CTAs per SM when every warp keeps at least 2 stages in half the shared memory,
  // otherwise one CTA with up to 3 stages per warp.
  static constexpr int HALF = 113 * 1024 - 1024 - COMB - PREFIX - 256;
  static constexpr int FULL = 226 * 1024 - 1024 - COMB - PREFIX - 256;
  static constexpr int PW_HALF = HALF / (2 * STAGE) / WPH;
  static constexpr int PW_FULL = FULL / (2 * STAGE) / WPH;
  static constexpr int PW = DEEP ? (PW_FULL > 6 ? 6 : PW_FULL)
                                 : (PW_HALF >= 2 ? (PW_HALF > 3 ? 3 : PW_HALF) : (PW_FULL > 3 ? 3 : PW_FULL));
  static constexpr int S = WPH * PW;
  static constexpr int RING = 2 * S * STAGE;
  static constexpr int SMEM = 1024 + RING + COMB + 2 * S * 8 + PREFIX;
  static constexpr int MIN_BLOCKS = 2 * (SMEM + 1024) <= 228 * 1024 ? 2 : 1;  // CTAs per SM to plan registers for
  static_assert(PW >= 2, "ring too shallow");
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
  int4* desc;        // [ctas] split sequence owned by each CTA: (sequence, pieces, first slot) or -1
  float* partials;  // [ctas][2][NH][RK][D + 4]: (m, l, pad, pad, O) per row
  int64_t out_sb, out_sh, q_sb, q_sh, kv_sb, kv_sh, table_stride;
  int32_t table_rows, table_cols;
  int32_t batch, group, layer, nbt, inputs_ready;
  float scale_log2;
};

// Largest b in [0, n) with p[b] <= t (p non-decreasing, p[0] = 0 <= t).
__device__ inline int seq_of(const int* p, int n, int t) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ inline void named_bar(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ inline void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}

template <typename T, int D, int NH, int RK, bool DEEP>
__global__ void __launch_bounds__(kThreads, DecodeShape<D, NH, RK, DEEP>::MIN_BLOCKS) decode_kernel(const __grid_constant__ CUtensorMap tmap_k,
                                                          const __grid_constant__ CUtensorMap tmap_v,
                                                          const DecodeParams p) {
  using S = DecodeShape<D, NH, RK, DEEP>;
  constexpr int TILE = S::TILE, STAGE = S::STAGE, NS = S::S, WPH = S::WPH, PW = S::PW, DP = S::DP;
  constexpr int WC = S::WARP_COMB;
  constexpr int ROW = D + 4;          // partial row: m, l, 2 pad floats, O[D] (O 16-byte aligned)
  constexpr int SLOT = RK * ROW;      // floats of one partial state of one head
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring_k = smem;
  uint8_t* ring_v = smem + NS * STAGE;
  float* comb = reinterpret_cast<float*>(smem + S::RING);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::RING + S::COMB);
  uint64_t* empty = full + NS;
  int* sP = reinterpret_cast<int*>(empty + NS);  // [batch + 1] block prefix sums
  int* sCtx = sP + kMaxBatch + 1;                // [batch] clamped context lengths
  int* sRow = sCtx + kMaxBatch + 1;              // [batch] block-table row of each sequence
  __shared__ int s_bad;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g_lane = lane >> 2, t4 = lane & 3;
  const int B = p.batch, G = p.group;
  const int cap = p.table_cols * kBS;

  // With programmatic dependent launch this CTA may start while the previous kernel in
  // the stream drains; let the next kernel launch early too. Everything the previous
  // kernel may have produced is read only after grid_dep_wait(). With inputs_ready the
  // caller guarantees that context lengths, table rows and the cached K/V were complete
  // before the previous kernel began, so the prologue, the block lookups and the first
  // ring fill run before the wait, overlapping the previous kernel's tail; q, the new
  // rows, the append, the output and the workspace still come after it.
  grid_dep_launch_dependents();
  if (!p.inputs_ready) grid_dep_wait();

  // Every thread fetches some context lengths and table rows (independent loads, one
  // round trip for the whole batch); warp 0 then scans them in shared memory.
  for (int i = tid; i < B; i += blockDim.x) {
    int ctx = p.context_lens[i];
    int row = p.seq_rows ? p.seq_rows[i] : i;
    if (ctx > cap) {
      report(p.status, PKV_ERR_OUT_OF_RANGE);
      ctx = cap;
    }
    if (row >= p.table_rows) {
      report(p.status, PKV_ERR_OUT_OF_RANGE);
      row = -1;
    }
    sCtx[i] = max(ctx, 0);
    sRow[i] = row;
  }
  __syncthreads();
  if (warp == 0) {  // prefix sums of the per-sequence block counts
    int carry = 0;
    for (int base = 0; base < B; base += 32) {
      const int i = base + lane;
      int v = i < B ? (sCtx[i] + kBS - 1) / kBS : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
      }
      if (i < B) sP[i + 1] = carry + v;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) sP[0] = 0;
  }
  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NH);  // one consumer warp per head releases each stage
    }
    fence_mbar_init();
    s_bad = 0;
  }
  __syncthreads();

  const int total = sP[B];
  const int ctas = min((int)gridDim.x, max(total, 1));  // every working CTA gets at least one tile
  const int g = blockIdx.x;
  if (g == 0) {  // sequences with nothing to attend to get zeros (the reference never asks for this)
    grid_dep_wait();
    for (int b = warp; b < B; b += kNC + 1) {
      if (sCtx[b] != 0) continue;
      T* o = reinterpret_cast<T*>(p.out) + b * p.out_sb;
      for (int e = lane; e < NH * G * D; e += 32) o[(e / D) * p.out_sh + e % D] = Dt<T>::from_f(0.f);
    }
  }
  if (g >= ctas) {  // no tiles: only say so to the merge kernel (after the previous one read its copy)
    if (tid == 0) {
      grid_dep_wait();
      p.desc[g] = make_int4(-1, 0, 0, 0);
    }
    return;
  }
  // Tile j of the run is consumed, for every head, by warp j % WPH of that head, whose
  // private stages are w * PW .. w * PW + PW - 1. A warp therefore waits on every phase
  // of its stages in order (an mbarrier parity wait is only unambiguous within one phase
  // of the barrier), and the previous use of tile j's stage is tile j - NS.
  auto stage_of = [](int j) { return (j % WPH) * PW + (j / WPH) % PW; };
  auto use_of = [](int j) { return (j / WPH) / PW; };
  const int t0 = (int)((int64_t)total * g / ctas);
  const int t1 = (int)((int64_t)total * (g + 1) / ctas);
  const int n = t1 - t0;
  const uint64_t deadline = global_ns() + kWaitBudgetNs;

  if (warp == kNC) {
    // ---------------------------------------------------------------- producer
    const uint64_t pol = policy_evict_first();
    auto lookup = [&](int j) -> int {  // block id of local tile j
      if (j >= n) return 0;
      const int t = t0 + j;
      const int b = seq_of(sP, B, t);
      const int i = t - sP[b];
      const int row = sRow[b];
      int blk = row >= 0 ? p.tables[row * p.table_stride + i] : p.nbt - 1;  // padding rows: scratch block
      if (blk < 0 || blk >= p.nbt) {
        report(p.status, PKV_ERR_OUT_OF_RANGE);
        blk = p.nbt - 1;
      }
      return blk;
    };
    int blk_next = lookup(lane);
    bool ok = true;
    for (int base = 0; base < n && ok; base += 32) {
      const int blk_cur = blk_next;
      blk_next = lookup(base + 32 + lane);  // in flight while this batch is issued
      const int cnt = min(32, n - base);
      for (int k = 0; k < cnt && ok; ++k) {
        const int blk = __shfl_sync(0xffffffffu, blk_cur, k);
        const int j = base + k;
        const int st = stage_of(j);
        if (j == NS) grid_dep_wait();  // before the consumers can release anything
        if (lane == 0) {
          if (j >= NS && !mbar_wait_until(&empty[st], (use_of(j) - 1) & 1, deadline)) {
            report(p.status, PKV_ERR_TIMEOUT);
            ok = false;
          }
          if (ok) {
            const int c4 = p.layer * p.nbt + blk;
            mbar_arrive_expect_tx(&full[st], 2 * STAGE);
            tma_load_5d(ring_k + st * STAGE, &tmap_k, 0, 0, 0, 0, c4, &full[st], pol);
            tma_load_5d(ring_v + st * STAGE, &tmap_v, 0, 0, 0, 0, c4, &full[st], pol);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
      }
    }
    if (n <= NS) grid_dep_wait();
    if (!ok) s_bad = 1;
  } else {
    // ---------------------------------------------------------------- consumers
    grid_dep_wait();  // q, the new rows, the output and the pool writes depend on earlier kernels
    // Every warp of a head walks the same pieces and meets the same named barriers, also
    // after a timed-out wait (then it skips waits and math), so no barrier is left short.
    const int h = warp / WPH, w = warp % WPH;
    float* head_comb = comb + h * WPH * WC;
    bool ok = true;
    // Q fragments of this head's query group (A operand, rows = query heads). The next
    // piece's are fetched while this piece runs, so a piece boundary does not wait on them.
    auto load_q = [&](int bq, uint32_t (&dst)[D / 16][4]) {
      const T* qb = reinterpret_cast<const T*>(p.q) + bq * p.q_sb + (int64_t)h * G * p.q_sh;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int c0 = kk * 16 + 2 * t4;
        dst[kk][0] = g_lane < G ? *reinterpret_cast<const uint32_t*>(qb + g_lane * p.q_sh + c0) : 0u;
        dst[kk][1] = g_lane + 8 < G ? *reinterpret_cast<const uint32_t*>(qb + (g_lane + 8) * p.q_sh + c0) : 0u;
        dst[kk][2] = g_lane < G ? *reinterpret_cast<const uint32_t*>(qb + g_lane * p.q_sh + c0 + 8) : 0u;
        dst[kk][3] = g_lane + 8 < G ? *reinterpret_cast<const uint32_t*>(qb + (g_lane + 8) * p.q_sh + c0 + 8) : 0u;
      }
    };
    uint32_t qa[D / 16][4];
    for (int b = seq_of(sP, B, t0); b < B && sP[b] < t1; ++b) {
      const int ja = max(t0, sP[b]) - t0, jb = min(t1, sP[b + 1]) - t0;
      if (ja >= jb) continue;  // an empty sequence
      const int ctx = sCtx[b];
      load_q(b, qa);
      const int append_blk = p.k_new ? (ctx - 1) / kBS : -1;
      float m_r[2] = {-INFINITY, -INFINITY};
      float l_r[2] = {0.f, 0.f};
      float o[D / 8][4];
#pragma unroll
      for (int jj = 0; jj < D / 8; ++jj) o[jj][0] = o[jj][1] = o[jj][2] = o[jj][3] = 0.f;

      for (int j = ja + ((w - ja) % WPH + WPH) % WPH; j < jb; j += WPH) {
        const int st = stage_of(j);
        if (ok && !mbar_wait_until(&full[st], use_of(j) & 1, deadline)) {
          report(p.status, PKV_ERR_TIMEOUT);
          ok = false;
        }
        if (ok) {
          uint8_t* kt = ring_k + st * STAGE + h * TILE;
          uint8_t* vt = ring_v + st * STAGE + h * TILE;
          const int i = t0 + j - sP[b];  // block index within the sequence
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
              const uint32_t kw = *reinterpret_cast<const uint32_t*>(kn + d0);
              const uint32_t vw = *reinterpret_cast<const uint32_t*>(vn + d0);
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
      // Merge the head's warps through shared memory.
      float* cm = head_comb + w * WC;
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
      const bool whole = sP[b] >= t0 && sP[b + 1] <= t1;
      const int slot_kind = sP[b] <= t0 ? 0 : 1;  // the run's first piece, else its last
      float* part = p.partials + ((int64_t)(g * 2 + slot_kind) * NH + h) * SLOT;
      T* outp = reinterpret_cast<T*>(p.out) + b * p.out_sb + (int64_t)h * G * p.out_sh;
      for (int it = w * 32 + lane; it < G * (D / 2); it += WPH * 32) {
        const int r = it / (D / 2), col = 2 * (it % (D / 2));
        float mm = -INFINITY;
#pragma unroll
        for (int ww = 0; ww < WPH; ++ww) mm = fmaxf(mm, head_comb[ww * WC + r]);
        float ll = 0.f, o0 = 0.f, o1 = 0.f;
#pragma unroll
        for (int ww = 0; ww < WPH; ++ww) {
          const float* c = head_comb + ww * WC;
          const float f = ex2(c[r] - mm);
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
      named_bar(1 + h, WPH * 32);  // the combine buffer is reused by the next piece
    }
    if (!ok) s_bad = 1;
  }
  __syncthreads();
  // Hand the split sequence whose first piece ends this run to the merge kernel: this CTA
  // owns it when the run's last tile belongs to a sequence that started inside the run and
  // continues past it. Every CTA rewrites its descriptor on every call.
  if (tid == 0) {
    int4 d = make_int4(-1, 0, 0, 0);
    const int b = seq_of(sP, B, t1 - 1);
    if (!s_bad && sP[b] >= t0 && sP[b + 1] > t1) {
      const int last_cta = (int)(((int64_t)sP[b + 1] * ctas - 1) / total);  // CTA of tile sP[b + 1] - 1
      d = make_int4(b, last_cta - g + 1, sP[b] == t0 ? 0 : 1, 0);
    }
    p.desc[g] = d;
  }
}

// Merges the pieces of every split sequence, one CTA per possible owner (the decode
// kernel's CTA g writes descriptor g). Pieces are combined in run order with the
// running-max rescaling of the flash step, so the result does not depend on timing.
// Each thread takes (head, row, 4 columns) items and loads up to 8 pieces' states at a
// time, all independent, so a merge of up to 8 pieces costs one round trip to L2.
constexpr int kMergeThreads = 512;

template <typename T, int D, int NH, int RK>
__global__ void __launch_bounds__(kMergeThreads) decode_merge_kernel(const DecodeParams p) {
  constexpr int ROW = D + 4;
  constexpr int SLOT = RK * ROW;
  grid_dep_launch_dependents();
  grid_dep_wait();  // the decode kernel's pieces and descriptors
  const int4 d = __ldcg(&p.desc[blockIdx.x]);
  if (d.x < 0) return;
  const int b = d.x, np = d.y, kind0 = d.z, first = blockIdx.x;
  const int G = p.group;
  const int items = NH * G * (D / 4);
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int c = (it % (D / 4)) * 4;
    const int r = (it / (D / 4)) % G;
    const int h = it / (G * (D / 4));
    float mx = -INFINITY, l = 0.f, a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    for (int q0 = 0; q0 < np; q0 += 8) {
      const int cnt = min(8, np - q0);
      float2 ml[8];
      float4 o[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (u < cnt) {
          const int q = q0 + u;
          const float* row = p.partials + ((int64_t)((first + q) * 2 + (q == 0 ? kind0 : 0)) * NH + h) * SLOT + r * ROW;
          ml[u] = __ldcg(reinterpret_cast<const float2*>(row));
          o[u] = __ldcg(reinterpret_cast<const float4*>(row + 4 + c));
        }
      }
      float mn = mx;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (u < cnt) mn = fmaxf(mn, ml[u].x);
      const float fo = mx == -INFINITY ? 0.f : ex2(mx - mn);
      l *= fo, a0 *= fo, a1 *= fo, a2 *= fo, a3 *= fo;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (u < cnt) {
          const float f = ml[u].x == -INFINITY ? 0.f : ex2(ml[u].x - mn);
          l += ml[u].y * f;
          a0 += o[u].x * f, a1 += o[u].y * f, a2 += o[u].z * f, a3 += o[u].w * f;
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

// Workspace: [descriptors: kMaxCtas int4][partials: ctas * 2 * NH * RK * (D + 4) float].
// Both are written before they are read within a call; nothing carries over between calls.
constexpr int kMaxCtas = 4 * 256;  // workspace is sized for up to 4 CTAs on each of up to 256 SMs
constexpr int64_t kPartialsOffset = (int64_t)kMaxCtas * 16;
int64_t ws_bytes(int ctas, int nh, int rk, int d) { return kPartialsOffset + (int64_t)ctas * 2 * nh * rk * (d + 4) * 4; }

// Tuning knobs, read once from the environment (0 / unset = built-in choice):
//   PKV_DECODE_CTAS_PER_SM  CTAs per SM (at most what the shared memory allows)
//   PKV_DECODE_PDL          0 = launch without programmatic stream serialization
//   PKV_DECODE_DEEP         1 = one CTA per SM with the deepest ring that fits
struct DecodeKnobs {
  int ctas_per_sm = 0, pdl = 1, deep = 0;
  DecodeKnobs() {
    auto env = [](const char* k, int dflt) {
      const char* v = getenv(k);
      return v && *v ? atoi(v) : dflt;
    };
    ctas_per_sm = env("PKV_DECODE_CTAS_PER_SM", 0);
    pdl = env("PKV_DECODE_PDL", 1);
    deep = env("PKV_DECODE_DEEP", 0);
  }
};
const DecodeKnobs& knobs() {
  static const DecodeKnobs k;
  return k;
}

template <typename T, int D, int NH, int RK, bool DEEP>
int launch_decode(const pkv_pool& pool, const DecodeParams& p0, void* workspace, int64_t workspace_bytes,
                  cudaStream_t stream) {
  using S = DecodeShape<D, NH, RK, DEEP>;
  static int per_sm = 0;
  if (per_sm == 0) {
    cudaError_t e = cudaFuncSetAttribute(decode_kernel<T, D, NH, RK, DEEP>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM);
    if (e != cudaSuccess) return cuda_status(e);
    int occ = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, decode_kernel<T, D, NH, RK, DEEP>, kThreads, S::SMEM);
    if (e != cudaSuccess) return cuda_status(e);
    per_sm = std::max(1, occ);
  }
  const int want = knobs().ctas_per_sm > 0 ? std::min(knobs().ctas_per_sm, per_sm) : per_sm;
  const int ctas = std::min(num_sms() * want, kMaxCtas);
  if (!workspace || workspace_bytes < ws_bytes(ctas, NH, RK, D)) return PKV_ERR_WORKSPACE;
  CUtensorMap tk, tv;
  if (!get_pool_maps(pool, &tk, &tv, NH)) return PKV_ERR_CUDA;
  DecodeParams p = p0;
  uint8_t* wsb = static_cast<uint8_t*>(workspace);
  p.desc = reinterpret_cast<int4*>(wsb);
  p.partials = reinterpret_cast<float*>(wsb + kPartialsOffset);
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
  const int st = cuda_status(cudaLaunchKernelEx(&cfg, decode_kernel<T, D, NH, RK, DEEP>, tk, tv, p));
  if (st != PKV_OK) return st;
  // The merge of split sequences: one small CTA per decode CTA, launched behind it (with
  // programmatic serialization it is resident early and waits on the decode grid).
  cfg.blockDim = dim3(kMergeThreads);
  cfg.dynamicSmemBytes = 0;
  return cuda_status(cudaLaunchKernelEx(&cfg, decode_merge_kernel<T, D, NH, RK>, p));
}

template <typename T, int D, int NH>
int launch_rows(const pkv_pool& pool, const DecodeParams& p, void* ws, int64_t wsb, cudaStream_t st) {
  if (knobs().deep)
    return p.group <= 8 ? launch_decode<T, D, NH, 8, true>(pool, p, ws, wsb, st)
                        : launch_decode<T, D, NH, 16, true>(pool, p, ws, wsb, st);
  return p.group <= 8 ? launch_decode<T, D, NH, 8, false>(pool, p, ws, wsb, st)
                      : launch_decode<T, D, NH, 16, false>(pool, p, ws, wsb, st);
}

template <typename T, int D>
int launch_heads(const pkv_pool& pool, const DecodeParams& p, void* ws, int64_t wsb, cudaStream_t st) {
  switch (pool.num_kv_heads) {
    case 1: return launch_rows<T, D, 1>(pool, p, ws, wsb, st);
    case 2: return launch_rows<T, D, 2>(pool, p, ws, wsb, st);
    case 4: return launch_rows<T, D, 4>(pool, p, ws, wsb, st);
    default: return PKV_ERR_UNSUPPORTED;
  }
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int64_t pkv_decode_workspace_bytes(int32_t batch, int32_t num_kv_heads, int32_t max_blocks_per_seq,
                                              int32_t block_size, int32_t head_dim, int32_t num_q_heads) {
  if (batch <= 0 || batch > kMaxBatch || num_kv_heads <= 0 || max_blocks_per_seq <= 0 || block_size != kBS ||
      (head_dim != 64 && head_dim != 128) || num_q_heads <= 0 || num_q_heads % num_kv_heads != 0)
    return 0;
  const int group = num_q_heads / num_kv_heads;
  return ws_bytes(kMaxCtas, num_kv_heads, group <= 8 ? 8 : 16, head_dim);
}

extern "C" int pkv_decode_attention(const pkv_pool* pool, int32_t layer, const pkv_tables* tables, int32_t batch,
                                    int32_t num_q_heads, void* out, int64_t out_stride_b, int64_t out_stride_h,
                                    const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k_new,
                                    const void* v_new, int64_t kv_stride_b, int64_t kv_stride_h,
                                    const int64_t* slot_mapping, const int32_t* context_lens, float scale,
                                    int32_t flags, void* workspace, int64_t workspace_bytes,
                                    int32_t* status_dev, pkv_stream_t stream) {
  if (!pool || !tables || !out || !q || !context_lens || !tables->block_tables) return PKV_ERR_INVALID_ARGUMENT;
  if (batch < 0 || layer < 0 || layer >= pool->num_layers) return PKV_ERR_INVALID_ARGUMENT;
  if (batch == 0) return PKV_OK;
  if (batch > kMaxBatch) return PKV_ERR_UNSUPPORTED;
  const int d = pool->head_dim, hkv = pool->num_kv_heads;
  if (pool->block_size != kBS || (d != 64 && d != 128)) return PKV_ERR_UNSUPPORTED;
  if (hkv <= 0 || num_q_heads <= 0 || num_q_heads % hkv != 0) return PKV_ERR_INVALID_ARGUMENT;
  const int group = num_q_heads / hkv;
  if (group > 16) return PKV_ERR_UNSUPPORTED;
  if ((k_new == nullptr) != (v_new == nullptr)) return PKV_ERR_INVALID_ARGUMENT;
  if (k_new && !slot_mapping) return PKV_ERR_INVALID_ARGUMENT;
  // 32-bit accesses to q, out and the new rows: even strides, 4-byte aligned bases.
  auto aligned4 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 3) == 0; };
  if (!aligned4(q) || !aligned4(out) || (k_new && (!aligned4(k_new) || !aligned4(v_new)))) return PKV_ERR_INVALID_ARGUMENT;
  if ((q_stride_b | q_stride_h | out_stride_b | out_stride_h) & 1) return PKV_ERR_INVALID_ARGUMENT;
  if (k_new && ((kv_stride_b | kv_stride_h) & 1)) return PKV_ERR_INVALID_ARGUMENT;
  if (tables->cols <= 0 || tables->rows <= 0) return PKV_ERR_INVALID_ARGUMENT;
  if (!tables->seq_rows && tables->rows < batch) return PKV_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return PKV_ERR_INVALID_ARGUMENT;

  DecodeParams p{};
  p.out = out;
  p.q = q;
  p.k_new = k_new;
  p.v_new = v_new;
  p.k_pool = pool->k;
  p.v_pool = pool->v;
  p.slot_mapping = slot_mapping;
  p.tables = tables->block_tables;
  p.seq_rows = tables->seq_rows;
  p.context_lens = context_lens;
  p.status = status_dev;
  p.out_sb = out_stride_b;
  p.out_sh = out_stride_h;
  p.q_sb = q_stride_b;
  p.q_sh = q_stride_h;
  p.kv_sb = kv_stride_b;
  p.kv_sh = kv_stride_h;
  p.table_stride = tables->stride;
  p.table_rows = tables->rows;
  p.table_cols = tables->cols;
  p.batch = batch;
  p.group = group;
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
