// Paged KV-cache data movement: decode append and copy-on-write tail forks.
//
// Both kernels are pure HBM streams: every thread moves one 16-byte vector,
// consecutive threads touch consecutive 16-byte chunks of one head row (append)
// or of one contiguous page prefix (fork), so each warp issues full 512-byte
// coalesced transactions.  All layers go in one launch (the reference issues one
// launch per layer and copy).
#include "common.cuh"

namespace be {

// ---------------------------------------------------------------------------
// Append (flashinfer.page.append_paged_kv_cache semantics, page_table.py:199-209)
// ---------------------------------------------------------------------------
template <int VEC_BYTES>
__global__ void __launch_bounds__(256) append_kernel(
    const char* __restrict__ k, const char* __restrict__ v, int64_t row_stride_b,
    int64_t in_layer_stride_b, const int32_t* __restrict__ batch_indices,
    const int32_t* __restrict__ positions, const int32_t* __restrict__ kv_indices,
    const int32_t* __restrict__ kv_indptr, int nnz, char* __restrict__ pool,
    int64_t pool_layer_stride_b, int num_layers, int num_pages, int page_size, int hkv,
    int row_bytes /* head_dim * elt */, int64_t total_chunks) {
  const int chunks_per_row = row_bytes / VEC_BYTES;          // per (token, head)
  const int chunks_per_tok = chunks_per_row * hkv;            // per token, one plane
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < total_chunks;
       c += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = c;
    const int cin = (int)(r % chunks_per_tok);
    r /= chunks_per_tok;
    const int plane = (int)(r % 2);
    r /= 2;
    const int i = (int)(r % nnz);
    const int layer = (int)(r / nnz);
    const int pos = positions[i];
    const int b = batch_indices[i];
    const int page = kv_indices[kv_indptr[b] + pos / page_size];
    if (page < 0 || page >= num_pages || pos < 0) {
      flag_range_error();
      continue;
    }
    const int head = cin / chunks_per_row;
    const int off = (cin % chunks_per_row) * VEC_BYTES;
    const char* src = (plane ? v : k) + layer * in_layer_stride_b + i * row_stride_b +
                      (int64_t)head * row_bytes + off;
    char* dst = pool + layer * pool_layer_stride_b +
                (((int64_t)page * 2 + plane) * page_size + pos % page_size) * hkv * row_bytes +
                (int64_t)head * row_bytes + off;
    if constexpr (VEC_BYTES == 16) {
      *reinterpret_cast<int4*>(dst) = __ldg(reinterpret_cast<const int4*>(src));
    } else if constexpr (VEC_BYTES == 4) {
      *reinterpret_cast<int*>(dst) = __ldg(reinterpret_cast<const int*>(src));
    } else {
      *reinterpret_cast<short*>(dst) = *reinterpret_cast<const short*>(src);
    }
  }
}

// One warp per (layer, token, plane) row: the token's K (or V) row of every KV
// head is one contiguous run of hkv * row_bytes in the input and in the page
// slot, so a row is a warp-wide memcpy of 16-byte vectors.  Each lane loads
// all its vectors of the row before storing any (up to ROW_UNROLL in flight per
// lane), and the row index is decomposed once per warp in 32-bit arithmetic.
constexpr int ROW_UNROLL = 8;
__global__ void __launch_bounds__(256) append_rows_kernel(
    const char* __restrict__ k, const char* __restrict__ v, int64_t row_stride_b,
    int64_t in_layer_stride_b, const int32_t* __restrict__ batch_indices,
    const int32_t* __restrict__ positions, const int32_t* __restrict__ kv_indices,
    const int32_t* __restrict__ kv_indptr, int nnz, char* __restrict__ pool,
    int64_t pool_layer_stride_b, int num_pages, int page_size, int tok_vecs /* hkv*row_bytes/16 */,
    int num_rows /* layers * nnz * 2 */) {
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  for (int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < num_rows;
       row += warps) {
    const int plane = row & 1;
    const int li = row >> 1;
    const int i = li % nnz, layer = li / nnz;
    int page = 0, pos = 0;
    if (lane == 0) {
      pos = positions[i];
      const int b = batch_indices[i];
      page = pos >= 0 ? kv_indices[kv_indptr[b] + pos / page_size] : -1;
    }
    page = __shfl_sync(0xffffffffu, page, 0);
    pos = __shfl_sync(0xffffffffu, pos, 0);
    if (page < 0 || page >= num_pages || pos < 0) {
      if (lane == 0) flag_range_error();
      continue;
    }
    const int4* src = reinterpret_cast<const int4*>((plane ? v : k) + layer * in_layer_stride_b +
                                                    i * row_stride_b);
    int4* dst = reinterpret_cast<int4*>(
        pool + layer * pool_layer_stride_b +
        (((int64_t)page * 2 + plane) * page_size + pos % page_size) * (int64_t)tok_vecs * 16);
    for (int c0 = 0; c0 < tok_vecs; c0 += 32 * ROW_UNROLL) {
      int4 buf[ROW_UNROLL];
#pragma unroll
      for (int u = 0; u < ROW_UNROLL; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < tok_vecs) buf[u] = __ldg(src + c);
      }
#pragma unroll
      for (int u = 0; u < ROW_UNROLL; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < tok_vecs) dst[c] = buf[u];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Fork: tokens [0, len) of K and V, page src -> page dst, every layer.
// In one page plane the first `len` tokens are one contiguous run of
// len * hkv * head_dim elements, so each (copy, layer, plane) is a memcpy.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) fork_kernel(
    char* __restrict__ pool, int64_t pool_layer_stride_b, int num_layers, int num_pages,
    int64_t plane_bytes, const int32_t* __restrict__ src_pages,
    const int32_t* __restrict__ dst_pages, const int32_t* __restrict__ lens, int64_t tok_bytes,
    int num_segs) {
  // one CTA per (copy, layer, plane) segment at a time (grid-stride); every thread
  // loads all of its <= ROW_UNROLL vectors of the segment before storing them
  for (int seg = blockIdx.x; seg < num_segs; seg += gridDim.x) {
    const int plane = seg & 1;
    const int layer = (seg >> 1) % num_layers;
    const int j = (seg >> 1) / num_layers;
    const int s = src_pages[j], d = dst_pages[j];
    const int n16 = (int)((lens[j] * tok_bytes) >> 4);
    if (s < 0 || s >= num_pages || d < 0 || d >= num_pages) {
      if (threadIdx.x == 0) flag_range_error();
      continue;
    }
    const int4* s4 = reinterpret_cast<const int4*>(pool + layer * pool_layer_stride_b +
                                                   ((int64_t)s * 2 + plane) * plane_bytes);
    int4* d4 = reinterpret_cast<int4*>(pool + layer * pool_layer_stride_b +
                                       ((int64_t)d * 2 + plane) * plane_bytes);
    for (int c0 = 0; c0 < n16; c0 += 256 * ROW_UNROLL) {
      int4 buf[ROW_UNROLL];
#pragma unroll
      for (int u = 0; u < ROW_UNROLL; ++u) {
        const int c = c0 + u * 256 + threadIdx.x;
        if (c < n16) buf[u] = __ldg(s4 + c);
      }
#pragma unroll
      for (int u = 0; u < ROW_UNROLL; ++u) {
        const int c = c0 + u * 256 + threadIdx.x;
        if (c < n16) d4[c] = buf[u];
      }
    }
  }
}

}  // namespace be

using namespace be;

extern "C" int be_append_paged_kv(const void* append_key, const void* append_value,
                                  int64_t row_stride, int64_t input_layer_stride,
                                  const int32_t* batch_indices, const int32_t* positions,
                                  const int32_t* kv_indices, const int32_t* kv_indptr, int nnz,
                                  void* paged_kv_cache, int64_t pool_layer_stride, int num_layers,
                                  int num_pages, int page_size, int num_kv_heads, int head_dim,
                                  int dtype, void* stream) {
  if (nnz < 0 || num_layers < 1 || page_size < 1 || num_kv_heads < 1 || head_dim < 1 ||
      dtype < BE_F32 || dtype > BE_BF16) {
    set_error("be_append_paged_kv: invalid shape or dtype");
    return BE_EINVAL;
  }
  if (nnz == 0) return BE_OK;
  if (!append_key || !append_value || !batch_indices || !positions || !kv_indices || !kv_indptr ||
      !paged_kv_cache) {
    set_error("be_append_paged_kv: null pointer");
    return BE_EINVAL;
  }
  const int elt = dtype_size(dtype);
  const int row_bytes = head_dim * elt;
  const int64_t rs = row_stride * elt, ls = input_layer_stride * elt, ps = pool_layer_stride * elt;
  auto aligned = [](uintptr_t x, int a) { return (x % a) == 0; };
  int vec = 2;
  for (int a : {16, 4}) {
    if (aligned((uintptr_t)append_key, a) && aligned((uintptr_t)append_value, a) &&
        aligned((uintptr_t)paged_kv_cache, a) && rs % a == 0 && ls % a == 0 && ps % a == 0 &&
        row_bytes % a == 0) {
      vec = a;
      break;
    }
  }
  const int64_t chunks = (int64_t)num_layers * nnz * 2 * num_kv_heads * (row_bytes / vec);
  const int threads = 256;
  const int64_t want = (chunks + threads - 1) / threads;
  const int blocks = (int)(want < 148 * 16 ? want : 148 * 16);
  cudaStream_t st = (cudaStream_t)stream;
  auto* k = (const char*)append_key;
  auto* v = (const char*)append_value;
  auto* pool = (char*)paged_kv_cache;
  const int64_t tok_b = (int64_t)num_kv_heads * row_bytes;
  const int64_t rows = (int64_t)num_layers * nnz * 2;
  if (vec == 16 && tok_b / 16 <= (1 << 20) && rows < (1ll << 31)) {
    // 8 warps per CTA, one row per warp, grid capped at 16 CTAs per SM
    const int64_t want_r = (rows + 7) / 8;
    const int blocks_r = (int)(want_r < 148 * 16 ? want_r : 148 * 16);
    append_rows_kernel<<<blocks_r, 256, 0, st>>>(k, v, rs, ls, batch_indices, positions,
                                                 kv_indices, kv_indptr, nnz, pool, ps, num_pages,
                                                 page_size, (int)(tok_b / 16), (int)rows);
  } else if (vec == 16)
    append_kernel<16><<<blocks, threads, 0, st>>>(k, v, rs, ls, batch_indices, positions, kv_indices,
                                                  kv_indptr, nnz, pool, ps, num_layers, num_pages,
                                                  page_size, num_kv_heads, row_bytes, chunks);
  else if (vec == 4)
    append_kernel<4><<<blocks, threads, 0, st>>>(k, v, rs, ls, batch_indices, positions, kv_indices,
                                                 kv_indptr, nnz, pool, ps, num_layers, num_pages,
                                                 page_size, num_kv_heads, row_bytes, chunks);
  else
    append_kernel<2><<<blocks, threads, 0, st>>>(k, v, rs, ls, batch_indices, positions, kv_indices,
                                                 kv_indptr, nnz, pool, ps, num_layers, num_pages,
                                                 page_size, num_kv_heads, row_bytes, chunks);
  BE_LAUNCH_CHECK();
  return BE_OK;
}

extern "C" int be_fork_tail_copy(void* paged_kv_cache, int64_t pool_layer_stride, int num_layers,
                                 int num_pages, int page_size, int num_kv_heads, int head_dim,
                                 int dtype, const int32_t* src_pages, const int32_t* dst_pages,
                                 const int32_t* lens, int num_copies, void* stream) {
  if (num_copies < 0 || num_layers < 1 || page_size < 1 || num_kv_heads < 1 || head_dim < 1 ||
      dtype < BE_F32 || dtype > BE_BF16) {
    set_error("be_fork_tail_copy: invalid shape or dtype");
    return BE_EINVAL;
  }
  if (num_copies == 0) return BE_OK;
  const int elt = dtype_size(dtype);
  const int64_t tok_bytes = (int64_t)num_kv_heads * head_dim * elt;
  if (tok_bytes % 16 || ((uintptr_t)paged_kv_cache % 16) || (pool_layer_stride * elt) % 16) {
    set_error("be_fork_tail_copy: pool rows must be 16-byte aligned (kv_heads*head_dim*elt %% 16)");
    return BE_EINVAL;
  }
  const int64_t segs = (int64_t)num_copies * num_layers * 2;
  if (segs >= (1ll << 31)) {
    set_error("be_fork_tail_copy: too many copies x layers (%lld segments)", (long long)segs);
    return BE_EINVAL;
  }
  if (((int64_t)page_size * tok_bytes) >> 4 >= (1ll << 31)) {
    set_error("be_fork_tail_copy: page too large");
    return BE_EINVAL;
  }
  const int grid = (int)(segs < 148 * 8 ? segs : 148 * 8);
  fork_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
      (char*)paged_kv_cache, pool_layer_stride * elt, num_layers, num_pages, page_size * tok_bytes,
      src_pages, dst_pages, lens, tok_bytes, (int)segs);
  BE_LAUNCH_CHECK();
  return BE_OK;
}

extern "C" int be_device_status(int* out, void* stream) {
  BE_CUDA_CHECK(cudaMemcpyFromSymbolAsync(out, g_device_status, sizeof(int), 0,
                                          cudaMemcpyDeviceToHost, (cudaStream_t)stream));
  BE_CUDA_CHECK(cudaStreamSynchronize((cudaStream_t)stream));
  return BE_OK;
}

extern "C" int be_device_status_clear(void* stream) {
  static const int zero = 0;
  BE_CUDA_CHECK(cudaMemcpyToSymbolAsync(g_device_status, &zero, sizeof(int), 0,
                                        cudaMemcpyHostToDevice, (cudaStream_t)stream));
  return BE_OK;
}

// ---------------------------------------------------------------------------
// Fork with the copy list in device memory (for a captured decode step):
// list = [count | src[cap] | dst[cap] | len[cap]].  A fixed grid strides over
// the count * layers * 2 (copy, layer, plane) segments, so one launch shape
// serves every step; a step without copies costs one wave of empty CTAs.
// ---------------------------------------------------------------------------
namespace be {

__global__ void __launch_bounds__(256) fork_list_kernel(
    char* __restrict__ pool, int64_t pool_layer_stride_b, int num_layers, int num_pages,
    int page_size, int64_t tok_bytes, const int32_t* __restrict__ list, int cap) {
  const int count = min(max(list[0], 0), cap);
  const int32_t* src_pages = list + 1;
  const int32_t* dst_pages = list + 1 + cap;
  const int32_t* lens = list + 1 + 2 * cap;
  const int64_t plane_bytes = page_size * tok_bytes;
  const int64_t nseg = (int64_t)count * num_layers * 2;
  for (int64_t seg = blockIdx.x; seg < nseg; seg += gridDim.x) {
    const int plane = (int)(seg & 1);
    const int64_t jl = seg >> 1;
    const int layer = (int)(jl % num_layers);
    const int j = (int)(jl / num_layers);
    const int s = src_pages[j], d = dst_pages[j], len = lens[j];
    if (s < 0 || s >= num_pages || d < 0 || d >= num_pages || len < 0 || len > page_size) {
      if (threadIdx.x == 0) flag_range_error();
      continue;
    }
    const int4* s4 = reinterpret_cast<const int4*>(
        pool + layer * pool_layer_stride_b + ((int64_t)s * 2 + plane) * plane_bytes);
    int4* d4 = reinterpret_cast<int4*>(pool + layer * pool_layer_stride_b +
                                       ((int64_t)d * 2 + plane) * plane_bytes);
    const int n16 = (int)((len * tok_bytes) >> 4);
    for (int c = threadIdx.x; c < n16; c += blockDim.x) d4[c] = __ldg(s4 + c);
  }
}

}  // namespace be

extern "C" int be_fork_tail_copy_list(void* paged_kv_cache, int64_t pool_layer_stride,
                                      int num_layers, int num_pages, int page_size,
                                      int num_kv_heads, int head_dim, int dtype,
                                      const int32_t* copy_list, int cap, int num_sms,
                                      void* stream) {
  using namespace be;
  if (!paged_kv_cache || !copy_list || cap < 0 || num_layers < 1 || page_size < 1 ||
      num_kv_heads < 1 || head_dim < 1 || dtype < BE_F32 || dtype > BE_BF16) {
    set_error("be_fork_tail_copy_list: invalid arguments");
    return BE_EINVAL;
  }
  const int elt = dtype_size(dtype);
  const int64_t tok_bytes = (int64_t)num_kv_heads * head_dim * elt;
  if (tok_bytes % 16 || ((uintptr_t)paged_kv_cache % 16) || (pool_layer_stride * elt) % 16) {
    set_error("be_fork_tail_copy_list: pool rows must be 16-byte aligned");
    return BE_EINVAL;
  }
  const int grid = 4 * (num_sms > 0 ? num_sms : 148);
  fork_list_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
      (char*)paged_kv_cache, pool_layer_stride * elt, num_layers, num_pages, page_size, tok_bytes,
      copy_list, cap);
  BE_LAUNCH_CHECK();
  return BE_OK;
}
