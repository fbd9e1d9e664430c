// be_attn_run: dispatch between the TMA-fed kernel (bf16/fp16, page lists,
// page size 16, head_dim 64/128), the cp.async tensor-core kernel (other
// 2-byte cases, slot lists) and the CUDA-core kernel (fp32), then the LSE merge.
#include "common.cuh"

namespace be {

template <typename T>
int launch_all(const AttnParams& p, const be_attn_plan_info* info, const int32_t* plan, int D,
               cudaStream_t st) {
  if (p.n_work > 0) {
    int rc = BE_OK;
    if constexpr (sizeof(T) == 2) {
      const bool tma_ok = !info->any_slots && info->page_size == 16 && (D == 128 || D == 64) &&
                          !force_cp_async();
      if (tma_ok) {
        CUtensorMap map;
        rc = get_pool_map(p.pool, p.num_pages, p.page_size, p.hkv, D, DT<T>::id, &map);
        if (rc != BE_OK) return rc;
        const int cs = pick_cluster(info, p.hkv, p.page_size);
        // wide tiles (shared prefixes) on tcgen05 when their chunks fit TMEM/smem
        const bool umma = umma_enabled() && p.n_wide > 0 && info->max_wide_tokens <= UM_MAX_TOK &&
                          ((uintptr_t)p.out % 16 == 0) && (p.out_row_stride % 8 == 0);
        int w0 = 0;
        if (umma) {
          rc = D == 128 ? launch_umma<T, 128>(p, map, st) : launch_umma<T, 64>(p, map, st);
          if (rc != BE_OK) return rc;
          w0 = p.n_wide;
        }
        if (p.n_work > w0)
          rc = D == 128 ? launch_tma<T, 128>(p, map, cs, w0, st)
                        : launch_tma<T, 64>(p, map, cs, w0, st);
      } else if (D == 128) rc = launch_tc<T, 128>(p, st);
      else if (D == 64) rc = launch_tc<T, 64>(p, st);
      else {
        dim3 grid(p.n_work, p.hkv);
        attn_simt_kernel<T><<<grid, 128, 0, st>>>(p, D);
        BE_LAUNCH_CHECK();
      }
    } else {
      dim3 grid(p.n_work, p.hkv);
      attn_simt_kernel<T><<<grid, 128, 0, st>>>(p, D);
      BE_LAUNCH_CHECK();
    }
    if (rc != BE_OK) return rc;
  }
  if (info->n_merge > 0) {
    const int items = info->n_merge * p.hq;
    merge_kernel<T><<<(items + 3) / 4, 128, 0, st>>>(
        plan + info->off_merge_q, plan + info->off_merge_ptr, plan + info->off_merge_parts,
        info->n_merge, p.mid_o, p.mid_lse, p.hq, D, p.out, p.out_row_stride, p.lse);
    BE_LAUNCH_CHECK();
  }
  return BE_OK;
}

}  // namespace be

using namespace be;

extern "C" int be_attn_run(const int32_t* plan_dev, const be_attn_plan_info* info, const void* q,
                           int64_t q_row_stride, const void* paged_kv_cache, int num_pages,
                           int num_qo_heads, int num_kv_heads, int head_dim, int dtype,
                           float sm_scale, void* out, int64_t out_row_stride, float* lse,
                           float* mid_o, float* mid_lse, const int32_t* kv_list_override,
                           void* stream) {
  if (!plan_dev || !info || !q || !paged_kv_cache || !out) {
    set_error("be_attn_run: null pointer");
    return BE_EINVAL;
  }
  if (num_kv_heads < 1 || num_qo_heads % num_kv_heads || head_dim < 8 || head_dim > 256 ||
      head_dim % 8 || dtype < BE_F32 || dtype > BE_BF16) {
    set_error("be_attn_run: bad head configuration (Hq %d, Hkv %d, D %d)", num_qo_heads,
              num_kv_heads, head_dim);
    return BE_EINVAL;
  }
  if (info->group_size != num_qo_heads / num_kv_heads) {
    set_error("be_attn_run: plan group size %d != Hq/Hkv %d", info->group_size,
              num_qo_heads / num_kv_heads);
    return BE_EINVAL;
  }
  if (info->n_parts > 0 && (!mid_o || !mid_lse)) {
    set_error("be_attn_run: plan needs %d partial rows but mid_o/mid_lse is null", info->n_parts);
    return BE_EINVAL;
  }
  if (dtype != BE_F32 && (((uintptr_t)q | (uintptr_t)paged_kv_cache) % 16 ||
                          (q_row_stride * 2) % 16)) {
    set_error("be_attn_run: q and the pool must be 16-byte aligned (q_row_stride %% 8 == 0)");
    return BE_EINVAL;
  }
  AttnParams p;
  p.work = reinterpret_cast<const Work*>(plan_dev + info->off_work);
  p.qlist = plan_dev + info->off_qlist;
  p.kvlist = kv_list_override ? kv_list_override : plan_dev + info->off_kvlist;
  p.q = (const char*)q;
  p.q_row_stride = q_row_stride;
  p.pool = (const char*)paged_kv_cache;
  p.num_pages = num_pages;
  p.page_size = info->page_size;
  p.hq = num_qo_heads;
  p.hkv = num_kv_heads;
  p.g = num_qo_heads / num_kv_heads;
  p.scale_log2 = sm_scale * kLog2e;
  p.out = (char*)out;
  p.out_row_stride = out_row_stride;
  p.lse = lse;
  p.mid_o = mid_o;
  p.mid_lse = mid_lse;
  p.n_work = info->n_work;
  p.n_wide = info->n_work_wide;
  {
    const char* e = getenv("BE_ATTN_DEBUG");
    p.debug = e ? atoi(e) : 0;
  }
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case BE_BF16: return launch_all<__nv_bfloat16>(p, info, plan_dev, head_dim, st);
    case BE_F16: return launch_all<__half>(p, info, plan_dev, head_dim, st);
    default: return launch_all<float>(p, info, plan_dev, head_dim, st);
  }
}
