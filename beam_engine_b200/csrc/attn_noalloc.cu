// be_attn_run_noalloc: paged attention for callers that cannot allocate device
// memory.
//
// be_attn_run needs two scratch buffers from its caller (mid_o / mid_lse, the
// partial rows that the LSE merge combines).  Some hosts of this library cannot
// provide them: code embedded in another runtime that owns every device
// allocation (a serving process whose memory pool is carved up at start-up, a
// plugin that may only touch the tensors it is handed), or code running where a
// cudaMalloc would synchronise the device or break an allocation budget.  This
// entry point takes the same plan, inputs and outputs but keeps the partial
// rows in a fixed array that lives in the library itself and is never
// allocated at run time.
//
// The array below is file-scope device memory of BE_NOALLOC_SCRATCH_BYTES
// (16 MiB).  Every GPU that loads the library reserves it until the process
// exits.  Plans whose partial rows need more than that are rejected.
namespace be {

constexpr size_t kNoAllocScratchBytes = BE_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch, looked up once per device.  In host
// code the symbol itself only names a host-side stand-in, so a kernel must be
// given this address, never &g_noalloc_scratch.
static int noalloc_scratch_address(void** out) {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  int dev = 0;
  BE_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) {
    set_error("be_attn_run_noalloc: device ordinal %d out of range", dev);
    return BE_EINVAL;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      set_error("be_attn_run_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return BE_ECUDA;
    }
    addr[dev] = p;
  }
  *out = addr[dev];
  return BE_OK;
}

}  // namespace be

extern "C" int be_attn_run_noalloc(const int32_t* plan_dev, const be_attn_plan_info* info,
                                   const void* q, int64_t q_row_stride, const void* paged_kv_cache,
                                   int num_pages, int num_qo_heads, int num_kv_heads, int head_dim,
                                   int dtype, float sm_scale, void* out, int64_t out_row_stride,
                                   float* lse, const int32_t* kv_list_override, void* stream) {
  using namespace be;
  if (!info) {
    set_error("be_attn_run_noalloc: null plan info");
    return BE_EINVAL;
  }
  if (num_qo_heads < 1 || head_dim < 1 || info->n_parts < 0) {
    set_error("be_attn_run_noalloc: invalid shape");
    return BE_EINVAL;
  }
  // mid_o: n_parts x Hq x D floats, then mid_lse: n_parts x Hq floats (256-byte aligned)
  const size_t o_bytes = (size_t)info->n_parts * num_qo_heads * head_dim * sizeof(float);
  const size_t o_pad = (o_bytes + 255) / 256 * 256;
  const size_t l_bytes = (size_t)info->n_parts * num_qo_heads * sizeof(float);
  if (o_pad + l_bytes > kNoAllocScratchBytes) {
    set_error("be_attn_run_noalloc: plan needs %zu bytes of partial rows (%d rows x %d heads x "
              "%d dims); the built-in scratch holds %zu bytes -- use be_attn_run with caller "
              "buffers or split the batch",
              o_pad + l_bytes, info->n_parts, num_qo_heads, head_dim, kNoAllocScratchBytes);
    return BE_ECAPACITY;
  }
  void* base = nullptr;
  int rc = noalloc_scratch_address(&base);
  if (rc != BE_OK) return rc;
  // Every partial row the plan names is written by its work item before the
  // merge reads it, so nothing in the shared array needs clearing.
  float* mid_o = reinterpret_cast<float*>(base);
  float* mid_lse = reinterpret_cast<float*>(reinterpret_cast<char*>(base) + o_pad);
  return be_attn_run(plan_dev, info, q, q_row_stride, paged_kv_cache, num_pages, num_qo_heads,
                     num_kv_heads, head_dim, dtype, sm_scale, out, out_row_stride, lse, mid_o,
                     mid_lse, kv_list_override, stream);
}
