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
// One CTA per (16-token query tile of one sequence, kv head) with one warp per
// query head of the GQA group: all warps share each K/V tile, which arrives by
// TMA into a 4-stage ring of swizzled shared memory. Each warp runs the same
// 16-key flash-attention step as the decode kernel (attn_tile.cuh).
#include "attn_tile.cuh"
#include "common.cuh"

namespace pkv {
namespace {

constexpr int kBS = 16;
constexpr int kStages = 4;
constexpr float kLog2e = 1.4426950408889634f;

template <int D> struct PrefillShape {
  static constexpr int TILE = kBS * D * 2;
  static constexpr int SMEM = 2 * kStages * TILE + kStages * 8 + 1024;
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
  int32_t group, layer, nbt;
  float scale_log2;
};

template <typename T, int D>
__global__ void __launch_bounds__(512) prefill_kernel(const __grid_constant__ CUtensorMap tmap_k,
                                                      const __grid_constant__ CUtensorMap tmap_v,
                                                      const PrefillParams p) {
  using S = PrefillShape<D>;
  constexpr int TILE = S::TILE;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * kStages * TILE);

  const int tile = blockIdx.x, head = blockIdx.y, s = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int tok0 = p.cu[s];
  const int n_new = p.cu[s + 1] - tok0;
  if (tile * 16 >= n_new) return;
  const int start = p.starts[s];
  const int rows_here = min(16, n_new - tile * 16);
  const int q_first = start + tile * 16;             // position of the tile's first query
  int kend = q_first + rows_here;                     // keys 0 .. kend-1 are visible to the tile
  if (kend > p.table_cols * kBS) {
    if (tid == 0) report(p.status, PKV_ERR_OUT_OF_RANGE);
    kend = p.table_cols * kBS;
  }
  const int nkb = (kend + kBS - 1) / kBS;
  int row = p.seq_rows ? p.seq_rows[s] : s;
  if (row < 0 || row >= p.table_rows) {
    if (tid == 0) report(p.status, PKV_ERR_OUT_OF_RANGE);
    row = -1;
  }
  const int32_t* table = row >= 0 ? p.tables + row * p.table_stride : nullptr;

  auto issue = [&](int i) {
    const int st = i % kStages;
    int blk = table ? table[i] : p.nbt - 1;
    if (blk < 0 || blk >= p.nbt) {
      report(p.status, PKV_ERR_OUT_OF_RANGE);
      blk = p.nbt - 1;
    }
    const int c4 = p.layer * p.nbt + blk;
    mbar_arrive_expect_tx(&full[st], 2 * TILE);
    // Default L2 policy: the tiles of a sequence are re-read by its other query tiles.
    tma_load_5d(smem + st * TILE, &tmap_k, 0, 0, 0, head, c4, &full[st]);
    tma_load_5d(smem + (kStages + st) * TILE, &tmap_v, 0, 0, 0, head, c4, &full[st]);
  };

  const uint64_t deadline = global_ns() + kWaitBudgetNs;
  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) mbar_init(&full[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    for (int i = 0; i < min(kStages, nkb); ++i) issue(i);
  }

  // Q fragments of this warp's query head for the tile's 16 tokens (rows past the sequence are zero).
  const int hq = head * p.group + warp;
  uint32_t qa[D / 16][4];
  {
    const T* qb = reinterpret_cast<const T*>(p.q) + (int64_t)(tok0 + tile * 16) * p.q_st + (int64_t)hq * p.q_sh;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const int c0 = kk * 16 + 2 * t4;
      qa[kk][0] = g < rows_here ? *reinterpret_cast<const uint32_t*>(qb + g * p.q_st + c0) : 0u;
      qa[kk][1] = g + 8 < rows_here ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * p.q_st + c0) : 0u;
      qa[kk][2] = g < rows_here ? *reinterpret_cast<const uint32_t*>(qb + g * p.q_st + c0 + 8) : 0u;
      qa[kk][3] = g + 8 < rows_here ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * p.q_st + c0 + 8) : 0u;
    }
  }

  float m_r[2] = {-INFINITY, -INFINITY};
  float l_r[2] = {0.f, 0.f};
  float o[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  bool ok = true;
  for (int i = 0; i < nkb; ++i) {
    const int st = i % kStages;
    if (ok && !mbar_wait_until(&full[st], (i / kStages) & 1, deadline)) {
      report(p.status, PKV_ERR_TIMEOUT);
      ok = false;
    }
    if (ok) {
      attend_tile16<T, D>(qa, smem_u32(smem + st * TILE), smem_u32(smem + (kStages + st) * TILE), i * kBS,
                          [q_first, rows_here](int r, int key) { return r < rows_here && key <= q_first + r; },
                          p.scale_log2, m_r, l_r, o);
    }
    __syncthreads();  // every warp is done with stage st
    if (tid == 0 && ok && i + kStages < nkb) issue(i + kStages);
  }
  finish_row_sums(l_r);
  if (!ok) return;

  T* ob = reinterpret_cast<T*>(p.out) + (int64_t)(tok0 + tile * 16) * p.out_st + (int64_t)hq * p.out_sh;
#pragma unroll
  for (int j = 0; j < D / 8; ++j) {
    const int col = 8 * j + 2 * t4;
    if (g < rows_here) {
      const float inv = 1.f / l_r[0];
      *reinterpret_cast<uint32_t*>(ob + g * p.out_st + col) = Dt<T>::pack(o[j][0] * inv, o[j][1] * inv);
    }
    if (g + 8 < rows_here) {
      const float inv = 1.f / l_r[1];
      *reinterpret_cast<uint32_t*>(ob + (g + 8) * p.out_st + col) = Dt<T>::pack(o[j][2] * inv, o[j][3] * inv);
    }
  }
}

template <typename T, int D>
int launch_prefill(const CUtensorMap& tk, const CUtensorMap& tv, const PrefillParams& p, int tiles, int hkv,
                   int seqs, cudaStream_t st) {
  using S = PrefillShape<D>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(prefill_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM);
    if (e != cudaSuccess) return cuda_status(e);
    configured = true;
  }
  dim3 grid(tiles, hkv, seqs);
  prefill_kernel<T, D><<<grid, 32 * p.group, S::SMEM, st>>>(tk, tv, p);
  return launch_status();
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
  if (!get_pool_maps(*pool, &tk, &tv)) return PKV_ERR_CUDA;
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
  const int tiles = (max_new_tokens + 15) / 16;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (pool->dtype == PKV_F16)
    return d == 64 ? launch_prefill<__half, 64>(tk, tv, p, tiles, hkv, num_seqs, st)
                   : launch_prefill<__half, 128>(tk, tv, p, tiles, hkv, num_seqs, st);
  if (pool->dtype == PKV_BF16)
    return d == 64 ? launch_prefill<__nv_bfloat16, 64>(tk, tv, p, tiles, hkv, num_seqs, st)
                   : launch_prefill<__nv_bfloat16, 128>(tk, tv, p, tiles, hkv, num_seqs, st);
  return PKV_ERR_UNSUPPORTED;
}
