// Paged decode attention for sm_100a, fused with the one-token KV append.
//
// Replaces, per layer and decode step, PagedDecodeContext.attend
// (engine/kv_cache.py:611-620): the index_put append, the gather of every
// sequence's blocks into a padded contiguous copy, and decode_attention's SDPA
// (engine/model.py:126-147). Here nothing is gathered: K/V blocks are read in
// place through the block table, each exactly once.
//
// Work split (split-K "flash decoding"): one CTA per (chunk of CB blocks,
// kv head, sequence). A chunk's K and V tiles (one 16 x head_dim tile per block
// and head) are all requested up front with 5-D TMA bulk tensor copies into
// 128B-swizzled shared memory, so each CTA keeps CB * 2 tiles in flight. Each
// warp then takes every NW-th block: S = Q K^T and O += P V on mma.sync
// m16n8k16 (fp32 accumulate), where the M=16 rows are the GQA group's query
// heads (the reference regroups head h to (h / group, h % group) the same way),
// so each K/V tile read from HBM serves the whole group. The softmax is the
// online (running max / running sum) form in base 2, with row reductions by
// warp shuffles inside each quad of lanes (attn_tile.cuh).
//
// Partial results of a sequence's chunks are combined by the last CTA to
// finish (an atomic ticket per (sequence, head); no CTA ever waits for
// another). Chunks are combined in chunk order, so the result does not depend
// on which CTA finishes last. A sequence with one chunk skips the workspace.
#include <algorithm>

#include "attn_tile.cuh"
#include "common.cuh"

namespace pkv {
namespace {

constexpr int kBS = 16;   // tokens per block handled by this kernel
constexpr int kNW = 4;    // warps per CTA
constexpr float kLog2e = 1.4426950408889634f;

template <int D> struct DecodeShape {
  static constexpr int CB = D == 64 ? 8 : 4;  // blocks per chunk (32 KB of K+V tiles per CTA)
  static constexpr int TILE = kBS * D * 2;     // bytes of one (block, head) tile
  static constexpr int MAXR = 16;              // rows of the mma tile
  static constexpr int DP = D + 4;             // padded row of the warp-combine buffer (no bank conflicts)
  static constexpr int COMBINE = 2 * kNW * MAXR * 4 + kNW * MAXR * DP * 4;
  static constexpr int BARS = (2 * CB * TILE > COMBINE ? 2 * CB * TILE : COMBINE);  // barrier offset
  static constexpr int SMEM = BARS + CB * 8 + 1024;  // + barriers + alignment slack
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
  int32_t* counters;
  float* ws_m;
  float* ws_l;
  float* ws_o;
  int64_t out_sb, out_sh, q_sb, q_sh, kv_sb, kv_sh, table_stride;
  int32_t table_rows, table_cols;
  int32_t batch, num_kv_heads, group, layer, nbt, max_chunks;
  float scale_log2;
};

// Rows of the M=16 tile that carry real query heads and are kept in the combine.
template <int D> __host__ __device__ constexpr int kept_rows(int group) { return group <= 8 ? 8 : 16; }

template <typename T, int D>
__global__ void __launch_bounds__(kNW * 32) decode_kernel(const __grid_constant__ CUtensorMap tmap_k,
                                                          const __grid_constant__ CUtensorMap tmap_v,
                                                          const DecodeParams p) {
  using S = DecodeShape<D>;
  constexpr int CB = S::CB;
  constexpr int TILE = S::TILE;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::BARS);
  __shared__ int s_last;

  const int chunk = blockIdx.x, head = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int G = p.group;
  const int max_ctx = p.table_cols * kBS;

  int ctx = p.context_lens[b];
  if (ctx > max_ctx) {
    if (chunk == 0 && tid == 0) report(p.status, PKV_ERR_OUT_OF_RANGE);
    ctx = max_ctx;
  }
  const int nblk = (ctx + kBS - 1) / kBS;
  const int nchunks = (nblk + CB - 1) / CB;
  if (ctx <= 0) {  // nothing to attend to: zeros (the reference never asks for this)
    if (chunk == 0) {
      T* o = reinterpret_cast<T*>(p.out) + b * p.out_sb;
      for (int i = tid; i < G * D; i += blockDim.x) o[(head * G + i / D) * p.out_sh + i % D] = Dt<T>::from_f(0.f);
    }
    return;
  }
  if (chunk >= nchunks) return;
  const int blk0 = chunk * CB;
  const int nb = min(CB, nblk - blk0);

  int row = p.seq_rows ? p.seq_rows[b] : b;
  if (row >= p.table_rows) {
    if (tid == 0) report(p.status, PKV_ERR_OUT_OF_RANGE);
    row = -1;
  }
  const int32_t* table = row >= 0 ? p.tables + row * p.table_stride : nullptr;

  const uint64_t deadline = global_ns() + kWaitBudgetNs;
  if (tid == 0) {
    for (int i = 0; i < nb; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0 && lane < nb) {
    int blk = table ? table[blk0 + lane] : p.nbt - 1;  // padding rows read the scratch block
    if (blk < 0 || blk >= p.nbt) {
      report(p.status, PKV_ERR_OUT_OF_RANGE);
      blk = p.nbt - 1;
    }
    const uint64_t pol = policy_evict_first();
    const int c4 = p.layer * p.nbt + blk;
    mbar_arrive_expect_tx(&bars[lane], 2 * TILE);
    tma_load_5d(smem + lane * TILE, &tmap_k, 0, 0, 0, head, c4, &bars[lane], pol);
    tma_load_5d(smem + (CB + lane) * TILE, &tmap_v, 0, 0, 0, head, c4, &bars[lane], pol);
  }

  // Q fragments (A operand, rows = the group's query heads), loaded while the tiles fly.
  uint32_t qa[D / 16][4];
  {
    const T* qb = reinterpret_cast<const T*>(p.q) + b * p.q_sb + (int64_t)head * G * p.q_sh;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const int c0 = kk * 16 + 2 * t4;
      qa[kk][0] = g < G ? *reinterpret_cast<const uint32_t*>(qb + g * p.q_sh + c0) : 0u;
      qa[kk][1] = g + 8 < G ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * p.q_sh + c0) : 0u;
      qa[kk][2] = g < G ? *reinterpret_cast<const uint32_t*>(qb + g * p.q_sh + c0 + 8) : 0u;
      qa[kk][3] = g + 8 < G ? *reinterpret_cast<const uint32_t*>(qb + (g + 8) * p.q_sh + c0 + 8) : 0u;
    }
  }

  // The fused append: the new token sits at position ctx - 1, in the last chunk.
  const bool append = p.k_new != nullptr && chunk == nchunks - 1;
  const int new_pos = ctx - 1;
  const int append_lb = append ? new_pos / kBS - blk0 : -1;

  float m_r[2] = {-INFINITY, -INFINITY};
  float l_r[2] = {0.f, 0.f};
  float o[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  bool timed_out = false;

  for (int lb = warp; lb < nb; lb += kNW) {
    if (!mbar_wait_until(&bars[lb], 0, deadline)) {
      timed_out = true;
      break;
    }
    uint8_t* kt = smem + lb * TILE;
    uint8_t* vt = smem + (CB + lb) * TILE;
    if (lb == append_lb) {
      // Put the new row into the staged tiles and write it to the pool at slot_mapping[b].
      const int off = new_pos % kBS;
      const int64_t slot = p.slot_mapping[b];
      const bool write = slot >= 0 && slot < (int64_t)p.nbt * kBS;
      if (slot >= (int64_t)p.nbt * kBS && lane == 0) report(p.status, PKV_ERR_OUT_OF_RANGE);
      const T* kn = reinterpret_cast<const T*>(p.k_new) + b * p.kv_sb + head * p.kv_sh;
      const T* vn = reinterpret_cast<const T*>(p.v_new) + b * p.kv_sb + head * p.kv_sh;
      const int64_t dst = (((int64_t)p.layer * p.nbt + (write ? slot / kBS : 0)) * p.num_kv_heads + head) * kBS * D +
                          (write ? slot % kBS : 0) * D;
#pragma unroll
      for (int w = lane; w < D / 2; w += 32) {
        const int d0 = 2 * w;
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
    const int key0 = (blk0 + lb) * kBS;
    attend_tile16<T, D>(qa, smem_u32(kt), smem_u32(vt), key0, [ctx](int, int key) { return key < ctx; },
                        p.scale_log2, m_r, l_r, o);
  }
  if (timed_out) report(p.status, PKV_ERR_TIMEOUT);
  // No copy may still be landing when the tiles' memory is reused below. On the normal
  // path every barrier has already completed and this is nb polls.
  if (tid == 0) {
    for (int i = 0; i < nb; ++i) {
      if (!mbar_wait_until(&bars[i], 0, deadline)) {
        report(p.status, PKV_ERR_TIMEOUT);
        break;
      }
    }
  }

  finish_row_sums(l_r);

  // Combine the warps through shared memory (the tiles are no longer needed).
  constexpr int MAXR = S::MAXR;
  constexpr int DP = S::DP;
  const int R = kept_rows<D>(G);
  __syncthreads();
  float* c_m = reinterpret_cast<float*>(smem);  // [kNW][MAXR]
  float* c_l = c_m + kNW * MAXR;                // [kNW][MAXR]
  float* c_o = c_l + kNW * MAXR;                // [kNW][R][DP]
  if (t4 == 0) {
    c_m[warp * MAXR + g] = m_r[0];
    c_l[warp * MAXR + g] = l_r[0];
    c_m[warp * MAXR + g + 8] = m_r[1];
    c_l[warp * MAXR + g + 8] = l_r[1];
  }
#pragma unroll
  for (int j = 0; j < D / 8; ++j) {
    const int col = 8 * j + 2 * t4;
    c_o[(warp * R + g) * DP + col] = o[j][0];
    c_o[(warp * R + g) * DP + col + 1] = o[j][1];
    if (R > 8) {
      c_o[(warp * R + g + 8) * DP + col] = o[j][2];
      c_o[(warp * R + g + 8) * DP + col + 1] = o[j][3];
    }
  }
  __syncthreads();

  const bool single = nchunks == 1;
  const int unit_idx = (b * p.num_kv_heads + head) * p.max_chunks + chunk;
  T* outp = reinterpret_cast<T*>(p.out) + b * p.out_sb + (int64_t)head * G * p.out_sh;
  // Each thread produces pairs of adjacent columns of the G x D result.
  for (int i = tid; i < G * (D / 2); i += blockDim.x) {
    const int r = i / (D / 2), col = 2 * (i % (D / 2));
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < kNW; ++w) mm = fmaxf(mm, c_m[w * MAXR + r]);
    float ll = 0.f, o0 = 0.f, o1 = 0.f;
#pragma unroll
    for (int w = 0; w < kNW; ++w) {
      const float f = ex2(c_m[w * MAXR + r] - mm);
      ll += c_l[w * MAXR + r] * f;
      o0 += c_o[(w * R + r) * DP + col] * f;
      o1 += c_o[(w * R + r) * DP + col + 1] * f;
    }
    if (single) {
      const float inv = 1.f / ll;
      *reinterpret_cast<uint32_t*>(outp + r * p.out_sh + col) = Dt<T>::pack(o0 * inv, o1 * inv);
    } else {
      float* wo = p.ws_o + ((int64_t)unit_idx * R + r) * D;
      __stcg(wo + col, o0);
      __stcg(wo + col + 1, o1);
      if (col == 0) {
        __stcg(p.ws_m + (int64_t)unit_idx * R + r, mm);
        __stcg(p.ws_l + (int64_t)unit_idx * R + r, ll);
      }
    }
  }
  if (single) return;

  // Last CTA of this (sequence, head) combines every chunk, in chunk order.
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    int* ctr = p.counters + b * p.num_kv_heads + head;
    const int ticket = atomicAdd(ctr, 1);
    s_last = ticket == nchunks - 1;
    if (s_last) *ctr = 0;  // ready for the next call
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int first = (b * p.num_kv_heads + head) * p.max_chunks;
  for (int i = tid; i < G * (D / 2); i += blockDim.x) {
    const int r = i / (D / 2), col = 2 * (i % (D / 2));
    float mm = -INFINITY;
    for (int c = 0; c < nchunks; ++c) mm = fmaxf(mm, __ldcg(p.ws_m + (int64_t)(first + c) * R + r));
    float ll = 0.f, o0 = 0.f, o1 = 0.f;
    for (int c = 0; c < nchunks; ++c) {
      const int64_t u = first + c;
      const float f = ex2(__ldcg(p.ws_m + u * R + r) - mm);
      ll += __ldcg(p.ws_l + u * R + r) * f;
      const float* wo = p.ws_o + (u * R + r) * D;
      o0 += __ldcg(wo + col) * f;
      o1 += __ldcg(wo + col + 1) * f;
    }
    const float inv = 1.f / ll;
    *reinterpret_cast<uint32_t*>(outp + r * p.out_sh + col) = Dt<T>::pack(o0 * inv, o1 * inv);
  }
}

// Workspace layout: [counters: kMaxTickets int32][m][l][o], where m and l are float
// [batch * Hkv * max_chunks * R] and o is float [batch * Hkv * max_chunks * R * D].
// The counter region has a fixed size, so calls with different batch sizes or
// table widths that share a workspace never see partial results where counters
// live (each counter is back at zero when its call ends).
constexpr int64_t kMaxTickets = 65536;

struct WsLayout {
  int64_t counters, m, l, o, total;
};

inline int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

WsLayout ws_layout(int batch, int hkv, int max_chunks, int rows, int d) {
  WsLayout w;
  const int64_t units = (int64_t)batch * hkv * max_chunks;
  w.counters = 0;
  w.m = kMaxTickets * 4;
  w.l = w.m + align256(units * rows * 4);
  w.o = w.l + align256(units * rows * 4);
  w.total = w.o + align256(units * rows * d * 4);
  return w;
}

int chunk_blocks(int d) { return d == 64 ? DecodeShape<64>::CB : DecodeShape<128>::CB; }

template <typename T, int D>
int launch_decode(const CUtensorMap& tk, const CUtensorMap& tv, const DecodeParams& p, int batch, int hkv,
                  cudaStream_t stream) {
  using S = DecodeShape<D>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(decode_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM);
    if (e != cudaSuccess) return cuda_status(e);
    configured = true;
  }
  dim3 grid(p.max_chunks, hkv, batch);
  decode_kernel<T, D><<<grid, kNW * 32, S::SMEM, stream>>>(tk, tv, p);
  return launch_status();
}

}  // namespace

bool get_pool_maps(const pkv_pool& pool, CUtensorMap* tk, CUtensorMap* tv);

}  // namespace pkv

using namespace pkv;

extern "C" int64_t pkv_decode_workspace_bytes(int32_t batch, int32_t num_kv_heads, int32_t max_blocks_per_seq,
                                              int32_t block_size, int32_t head_dim, int32_t num_q_heads) {
  if (batch <= 0 || num_kv_heads <= 0 || max_blocks_per_seq <= 0 || block_size != kBS ||
      (head_dim != 64 && head_dim != 128) || num_q_heads % num_kv_heads != 0)
    return 0;
  const int cb = chunk_blocks(head_dim);
  const int max_chunks = (max_blocks_per_seq + cb - 1) / cb;
  const int group = num_q_heads / num_kv_heads;
  return ws_layout(batch, num_kv_heads, max_chunks, group <= 8 ? 8 : 16, head_dim).total;
}

extern "C" int pkv_decode_attention(const pkv_pool* pool, int32_t layer, const pkv_tables* tables, int32_t batch,
                                    int32_t num_q_heads, void* out, int64_t out_stride_b, int64_t out_stride_h,
                                    const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k_new,
                                    const void* v_new, int64_t kv_stride_b, int64_t kv_stride_h,
                                    const int64_t* slot_mapping, const int32_t* context_lens, float scale,
                                    void* workspace, int64_t workspace_bytes, int32_t* status_dev,
                                    pkv_stream_t stream) {
  if (!pool || !tables || !out || !q || !context_lens || !tables->block_tables) return PKV_ERR_INVALID_ARGUMENT;
  if (batch < 0 || batch > 65535 || layer < 0 || layer >= pool->num_layers) return PKV_ERR_INVALID_ARGUMENT;
  if (batch == 0) return PKV_OK;
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
  if ((int64_t)batch * hkv > kMaxTickets) return PKV_ERR_UNSUPPORTED;

  const int cb = chunk_blocks(d);
  const int max_chunks = (tables->cols + cb - 1) / cb;
  const int rows = group <= 8 ? 8 : 16;
  const WsLayout ws = ws_layout(batch, hkv, max_chunks, rows, d);
  if (max_chunks > 1) {
    if (!workspace || workspace_bytes < ws.total) return PKV_ERR_WORKSPACE;
    if (reinterpret_cast<uintptr_t>(workspace) & 255) return PKV_ERR_INVALID_ARGUMENT;
  }
  CUtensorMap tk, tv;
  if (!get_pool_maps(*pool, &tk, &tv)) return PKV_ERR_CUDA;

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
  uint8_t* wsb = static_cast<uint8_t*>(workspace);
  p.counters = workspace ? reinterpret_cast<int32_t*>(wsb + ws.counters) : nullptr;
  p.ws_m = workspace ? reinterpret_cast<float*>(wsb + ws.m) : nullptr;
  p.ws_l = workspace ? reinterpret_cast<float*>(wsb + ws.l) : nullptr;
  p.ws_o = workspace ? reinterpret_cast<float*>(wsb + ws.o) : nullptr;
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
  p.num_kv_heads = hkv;
  p.group = group;
  p.layer = layer;
  p.nbt = pool->num_blocks_total;
  p.max_chunks = max_chunks;
  p.scale_log2 = scale * kLog2e;

  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (pool->dtype == PKV_F16) {
    return d == 64 ? launch_decode<__half, 64>(tk, tv, p, batch, hkv, st)
                   : launch_decode<__half, 128>(tk, tv, p, batch, hkv, st);
  }
  if (pool->dtype == PKV_BF16) {
    return d == 64 ? launch_decode<__nv_bfloat16, 64>(tk, tv, p, batch, hkv, st)
                   : launch_decode<__nv_bfloat16, 128>(tk, tv, p, batch, hkv, st);
  }
  return PKV_ERR_UNSUPPORTED;
}
