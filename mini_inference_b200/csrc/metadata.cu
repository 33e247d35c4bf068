// GPU builder for per-step paged-KV metadata, the device table mirror, and block copy.
//
// The reference rebuilds block tables, positions and write locations as Python
// lists every step and copies them to the device (engine/kv_cache.py:562-573,
// :597-609; engine/cuda_graphs.py:171-183). Here the block tables live on the
// device as a mirror indexed by slot, updated only where the host allocator
// changed them, and each step derives its metadata from it on the GPU.
#include <algorithm>

#include "common.cuh"

namespace pkv {
namespace {

__global__ void decode_meta_kernel(const int32_t* __restrict__ seq_rows, int32_t batch,
                                   const int32_t* __restrict__ tables, int64_t stride, int32_t rows, int32_t cols,
                                   const int32_t* __restrict__ lengths, int32_t bs, int32_t scratch,
                                   int64_t* __restrict__ positions, int64_t* __restrict__ slots,
                                   int32_t* __restrict__ ctx_lens, int32_t* status) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  int r = seq_rows[b];
  if (r >= rows) {
    report(status, PKV_ERR_OUT_OF_RANGE);
    r = -1;
  }
  if (r < 0) {  // CUDA-graph padding row: position 0 in the scratch block (engine/cuda_graphs.py:174-180)
    if (positions) positions[b] = 0;
    if (slots) slots[b] = (int64_t)scratch * bs;
    if (ctx_lens) ctx_lens[b] = 1;
    return;
  }
  const int32_t p = lengths[b];
  const int32_t col = p / bs;
  int64_t slot = -1;
  if (p < 0 || col >= cols) {
    report(status, PKV_ERR_OUT_OF_RANGE);
  } else {
    const int32_t blk = tables[r * stride + col];
    if (blk < 0) report(status, PKV_ERR_OUT_OF_RANGE);
    else slot = (int64_t)blk * bs + p % bs;
  }
  if (positions) positions[b] = p;
  if (slots) slots[b] = slot;
  if (ctx_lens) ctx_lens[b] = p + 1;
}

__global__ void prefill_meta_kernel(const int32_t* __restrict__ seq_rows, int32_t num_seqs,
                                    const int32_t* __restrict__ cu, const int32_t* __restrict__ starts,
                                    const int32_t* __restrict__ tables, int64_t stride, int32_t rows, int32_t cols,
                                    int32_t bs, int64_t total, int64_t* __restrict__ positions,
                                    int64_t* __restrict__ slots, int32_t* status) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= total) return;
  // sequence of token t: the last s with cu[s] <= t
  int lo = 0, hi = num_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= t) lo = mid; else hi = mid - 1;
  }
  const int s = lo;
  const int r = seq_rows ? seq_rows[s] : s;
  const int64_t pos = starts[s] + (t - cu[s]);
  if (positions) positions[t] = pos;
  int64_t slot = -1;
  if (r < 0 || r >= rows || pos / bs >= cols) {
    report(status, PKV_ERR_OUT_OF_RANGE);
  } else {
    const int32_t blk = tables[r * stride + pos / bs];
    if (blk < 0) report(status, PKV_ERR_OUT_OF_RANGE);
    else slot = (int64_t)blk * bs + pos % bs;
  }
  if (slots) slots[t] = slot;
}

__global__ void commit_kernel(const int32_t* __restrict__ seq_rows, int32_t batch, int32_t* lengths) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < batch && seq_rows[b] >= 0) lengths[seq_rows[b]] += 1;
}

__global__ void update_tables_kernel(int32_t* tables, int64_t stride, int32_t rows, int32_t cols,
                                     const int32_t* __restrict__ upd, int32_t n, int32_t* status) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int32_t r = upd[3 * i], c = upd[3 * i + 1], blk = upd[3 * i + 2];
  if (r < 0 || r >= rows || c < 0 || c >= cols) {
    report(status, PKV_ERR_OUT_OF_RANGE);
    return;
  }
  tables[r * stride + c] = blk;
}

// One thread per 16-byte vector of a (pair, layer, K|V) block image.
__global__ void copy_blocks_kernel(uint8_t* k, uint8_t* v, const int32_t* __restrict__ src,
                                   const int32_t* __restrict__ dst, int32_t n, int32_t layers, int32_t nbt,
                                   int64_t block_bytes, int32_t* status) {
  const int64_t vecs = block_bytes / 16;
  const int64_t total = (int64_t)n * layers * 2 * vecs;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t u = i % vecs;
    const int64_t rest = i / vecs;
    const int which = (int)(rest % 2);
    const int64_t l = (rest / 2) % layers;
    const int64_t pair = rest / (2 * (int64_t)layers);
    const int32_t s = src[pair], d = dst[pair];
    if (s < 0 || s >= nbt || d < 0 || d >= nbt) {
      if (u == 0) report(status, PKV_ERR_OUT_OF_RANGE);
      continue;
    }
    uint8_t* base = which ? v : k;
    const uint4 val = *reinterpret_cast<const uint4*>(base + ((l * nbt + s) * block_bytes) + u * 16);
    *reinterpret_cast<uint4*>(base + ((l * nbt + d) * block_bytes) + u * 16) = val;
  }
}

inline unsigned blocks_for(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int pkv_build_decode_metadata(const pkv_tables* tables, int32_t batch, const int32_t* lengths,
                                         int32_t block_size, int32_t scratch_block, int64_t* positions,
                                         int64_t* slot_mapping, int32_t* context_lens, int32_t* status_dev,
                                         pkv_stream_t stream) {
  if (!tables || !tables->block_tables || !tables->seq_rows || !lengths || block_size <= 0 || batch < 0)
    return PKV_ERR_INVALID_ARGUMENT;
  if (batch == 0) return PKV_OK;
  decode_meta_kernel<<<blocks_for(batch, 128), 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      tables->seq_rows, batch, tables->block_tables, tables->stride, tables->rows, tables->cols, lengths,
      block_size, scratch_block, positions, slot_mapping, context_lens, status_dev);
  return launch_status();
}

extern "C" int pkv_build_prefill_metadata(const pkv_tables* tables, int32_t num_seqs, const int32_t* cu_seqlens,
                                          const int32_t* starts, int32_t block_size, int64_t total_tokens,
                                          int64_t* positions, int64_t* slot_mapping, int32_t* status_dev,
                                          pkv_stream_t stream) {
  if (!tables || !tables->block_tables || !cu_seqlens || !starts || block_size <= 0 || num_seqs < 0 ||
      total_tokens < 0)
    return PKV_ERR_INVALID_ARGUMENT;
  if (total_tokens == 0 || num_seqs == 0) return PKV_OK;
  prefill_meta_kernel<<<blocks_for(total_tokens, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      tables->seq_rows, num_seqs, cu_seqlens, starts, tables->block_tables, tables->stride, tables->rows,
      tables->cols, block_size, total_tokens, positions, slot_mapping, status_dev);
  return launch_status();
}

extern "C" int pkv_commit_decode(const int32_t* seq_rows, int32_t batch, int32_t* lengths, pkv_stream_t stream) {
  if (!seq_rows || !lengths || batch < 0) return PKV_ERR_INVALID_ARGUMENT;
  if (batch == 0) return PKV_OK;
  commit_kernel<<<blocks_for(batch, 128), 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(seq_rows, batch,
                                                                                             lengths);
  return launch_status();
}

extern "C" int pkv_update_tables(int32_t* block_tables, int64_t table_stride, int32_t rows, int32_t cols,
                                 const int32_t* updates, int32_t n_updates, int32_t* status_dev,
                                 pkv_stream_t stream) {
  if (!block_tables || n_updates < 0 || (n_updates > 0 && !updates)) return PKV_ERR_INVALID_ARGUMENT;
  if (n_updates == 0) return PKV_OK;
  update_tables_kernel<<<blocks_for(n_updates, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      block_tables, table_stride, rows, cols, updates, n_updates, status_dev);
  return launch_status();
}

extern "C" int pkv_copy_blocks(const pkv_pool* pool, const int32_t* src, const int32_t* dst, int32_t n,
                               int32_t* status_dev, pkv_stream_t stream) {
  if (!pool || n < 0 || (n > 0 && (!src || !dst))) return PKV_ERR_INVALID_ARGUMENT;
  if (n == 0) return PKV_OK;
  const int64_t block_bytes = (int64_t)pool->num_kv_heads * pool->block_size * pool->head_dim * 2;
  if (block_bytes % 16) return PKV_ERR_UNSUPPORTED;
  const int64_t total = (int64_t)n * pool->num_layers * 2 * (block_bytes / 16);
  const unsigned grid = (unsigned)std::min<int64_t>((total + 255) / 256, 148 * 16);
  copy_blocks_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<uint8_t*>(pool->k), static_cast<uint8_t*>(pool->v), src, dst, n, pool->num_layers,
      pool->num_blocks_total, block_bytes, status_dev);
  return launch_status();
}
