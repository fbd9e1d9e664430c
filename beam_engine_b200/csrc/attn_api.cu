// be_attn_run / be_attn_run_fixed: dispatch between the tcgen05 kernel (wide
// tiles, bf16/fp16, page lists, page size 16, head_dim 64/128), the TMA-fed
// mma.sync kernel (narrow tiles), the cp.async tensor-core kernel (other 2-byte
// cases, slot lists) and the CUDA-core kernel (fp32), then the LSE merge.
#include "common.cuh"

namespace be {

struct Caps {                // grid sizes; fixed = true: counts come from the plan header
  int work, wide, merge, cluster;
  bool fixed;
  cudaStream_t side = nullptr;   // narrow tiles on this stream (fork / join by events)
  bool slots = false;            // fixed grids for plans with slot lists (tree plans)
};

// Fork / join events for the two-stream launch, one pair per device, created
// once (timing off).  Re-recording the same events is fine, also in a capture.
static int side_events(cudaEvent_t* fork, cudaEvent_t* join) {
  static std::mutex mu;
  static cudaEvent_t ev[64][2] = {};
  int dev = 0;
  BE_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) {
    set_error("device ordinal %d out of range", dev);
    return BE_EINVAL;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (!ev[dev][0]) {
    BE_CUDA_CHECK(cudaEventCreateWithFlags(&ev[dev][0], cudaEventDisableTiming));
    BE_CUDA_CHECK(cudaEventCreateWithFlags(&ev[dev][1], cudaEventDisableTiming));
  }
  *fork = ev[dev][0];
  *join = ev[dev][1];
  return BE_OK;
}

template <typename T>
int launch_all(const AttnParams& p, const be_attn_plan_info* info, const int32_t* plan, int D,
               const Caps& c, cudaStream_t st) {
  if (c.work > 0) {
    int rc = BE_OK;
    if constexpr (sizeof(T) == 2) {
      const bool tma_ok = (c.fixed ? !c.slots : (!info->any_slots && info->page_size == 16)) &&
                          p.page_size == 16 && (D == 128 || D == 64) && !force_cp_async();
      if (tma_ok) {
        CUtensorMap map;
        rc = get_pool_map(p.pool, p.num_pages, p.page_size, p.hkv, D, DT<T>::id, &map);
        if (rc != BE_OK) return rc;
        const int cs = c.fixed ? std::max(1, c.cluster) : pick_cluster(info, p.hkv, p.page_size);
        // wide tiles (shared prefixes) on tcgen05 when their chunks fit TMEM/smem
        const bool aligned = ((uintptr_t)p.out % 16 == 0) && (p.out_row_stride % 8 == 0);
        const bool umma = umma_enabled() && aligned && c.wide > 0 &&
                          (c.fixed || info->max_wide_tokens <= UM_MAX_TOK);
        const bool narrow = narrow_enabled() && p.hkv <= 8 && (umma || !c.fixed);
        int w0 = 0, n_items = c.work;
        if (umma && c.side) {   // fork point before the wide tiles: both start together
          cudaEvent_t f = nullptr, j = nullptr;
          rc = side_events(&f, &j);
          if (rc != BE_OK) return rc;
          BE_CUDA_CHECK(cudaEventRecord(f, st));
          BE_CUDA_CHECK(cudaStreamWaitEvent(c.side, f, 0));
        }
        if (umma) {
          rc = D == 128 ? (wide_enabled() ? launch_wide<T>(p, map, c.wide, st)
                                          : launch_umma<T, 128>(p, map, c.wide, st))
                        : launch_umma<T, 64>(p, map, c.wide, st);
          if (rc != BE_OK) return rc;
          w0 = c.fixed ? -1 : p.n_wide;
          n_items = c.fixed ? c.work : p.n_work - p.n_wide;
        } else if (narrow) {   // host-sized grid: wide items [0, n_wide) on the mma.sync kernel
          if (p.n_wide > 0) {
            rc = D == 128 ? launch_tma<T, 128>(p, map, cs, 0, p.n_wide, st)
                          : launch_tma<T, 64>(p, map, cs, 0, p.n_wide, st);
            if (rc != BE_OK) return rc;
          }
          w0 = p.n_wide;
          n_items = p.n_work - p.n_wide;
        }
        // narrow tiles: one CTA per item with every KV head (on the side stream
        // when there is one, so they overlap the tail of the wide tiles)
        if (n_items > 0 && narrow) {
          cudaStream_t ns = st;
          cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
          if (c.side && umma) {   // the side stream already waits on the fork point
            rc = side_events(&ev_fork, &ev_join);
            if (rc != BE_OK) return rc;
            ns = c.side;
          }
          rc = D == 128 ? launch_narrow<T, 128>(p, map, w0, n_items, ns)
                        : launch_narrow<T, 64>(p, map, w0, n_items, ns);
          if (ns != st) {
            BE_CUDA_CHECK(cudaEventRecord(ev_join, ns));
            BE_CUDA_CHECK(cudaStreamWaitEvent(st, ev_join, 0));
          }
        }
        else if (n_items > 0)
          rc = D == 128 ? launch_tma<T, 128>(p, map, cs, w0, n_items, st)
                        : launch_tma<T, 64>(p, map, cs, w0, n_items, st);
      } else if (D == 128) {
        rc = launch_tc<T, 128>(p, c.work, st);
      } else if (D == 64) {
        rc = launch_tc<T, 64>(p, c.work, st);
      } else {
        attn_simt_kernel<T><<<dim3(c.work, p.hkv), 128, 0, st>>>(p, D);
        BE_LAUNCH_CHECK();
      }
    } else {
      attn_simt_kernel<T><<<dim3(c.work, p.hkv), 128, 0, st>>>(p, D);
      BE_LAUNCH_CHECK();
    }
    if (rc != BE_OK) return rc;
  }
  if (c.merge > 0) {
    const int items = c.merge * p.hq;
    const bool dev = c.fixed;
    BE_CUDA_CHECK(launch_pdl(
        merge_kernel<T>, (items + 3) / 4, 128, 0, st,
        dev ? nullptr : plan + info->off_merge_q, dev ? nullptr : plan + info->off_merge_ptr,
        dev ? nullptr : plan + info->off_merge_parts, c.merge, (const float*)p.mid_o,
        (const float*)p.mid_lse, p.hq, D, p.out, p.out_row_stride, p.lse,
        dev ? plan : (const int32_t*)nullptr));
  }
  return BE_OK;
}

static int check_heads(int num_qo_heads, int num_kv_heads, int head_dim, int dtype) {
  if (num_kv_heads < 1 || num_qo_heads % num_kv_heads || head_dim < 8 || head_dim > 256 ||
      head_dim % 8 || dtype < BE_F32 || dtype > BE_BF16) {
    set_error("be_attn_run: bad head configuration (Hq %d, Hkv %d, D %d)", num_qo_heads,
              num_kv_heads, head_dim);
    return BE_EINVAL;
  }
  return BE_OK;
}

static void fill_params(AttnParams& p, const void* q, int64_t q_row_stride,
                        const void* paged_kv_cache, int num_pages, int page_size, int hq, int hkv,
                        float sm_scale, void* out, int64_t out_row_stride, float* lse,
                        float* mid_o, float* mid_lse) {
  p.q = (const char*)q;
  p.q_row_stride = q_row_stride;
  p.pool = (const char*)paged_kv_cache;
  p.num_pages = num_pages;
  p.page_size = page_size;
  p.hq = hq;
  p.hkv = hkv;
  p.g = hq / hkv;
  p.scale_log2 = sm_scale * kLog2e;
  p.out = (char*)out;
  p.out_row_stride = out_row_stride;
  p.lse = lse;
  p.mid_o = mid_o;
  p.mid_lse = mid_lse;
  const char* e = getenv("BE_ATTN_DEBUG");
  p.debug = e ? atoi(e) : 0;
  // BE_ATTN_WIDE_RUNS=1: the persistent wide kernel accumulates consecutive
  // chunks of one group before writing (bit 3 of the switches word)
  const char* r = getenv("BE_ATTN_WIDE_RUNS");
  if (r && r[0] == '1') p.debug |= 8;
}

template <typename... A>
static int dispatch(int dtype, A&&... a) {
  switch (dtype) {
    case BE_BF16: return launch_all<__nv_bfloat16>(a...);
    case BE_F16: return launch_all<__half>(a...);
    default: return launch_all<float>(a...);
  }
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
  int rc = check_heads(num_qo_heads, num_kv_heads, head_dim, dtype);
  if (rc) return rc;
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
  fill_params(p, q, q_row_stride, paged_kv_cache, num_pages, info->page_size, num_qo_heads,
              num_kv_heads, sm_scale, out, out_row_stride, lse, mid_o, mid_lse);
  p.hdr = nullptr;
  p.work = reinterpret_cast<const Work*>(plan_dev + info->off_work);
  p.qlist = plan_dev + info->off_qlist;
  p.kvlist = kv_list_override ? kv_list_override : plan_dev + info->off_kvlist;
  p.n_work = info->n_work;
  p.n_wide = info->n_work_wide;
  const Caps c{info->n_work, info->n_work_wide, info->n_merge, 0, false};
  return dispatch(dtype, p, info, plan_dev, head_dim, c, (cudaStream_t)stream);
}

extern "C" int be_attn_run_fixed(const int32_t* plan_dev, const be_attn_caps* caps, int page_size,
                                 const void* q, int64_t q_row_stride, const void* paged_kv_cache,
                                 int num_pages, int num_qo_heads, int num_kv_heads, int head_dim,
                                 int dtype, float sm_scale, void* out, int64_t out_row_stride,
                                 float* lse, float* mid_o, float* mid_lse,
                                 const int32_t* kv_list_override, void* stream) {
  if (!plan_dev || !caps || !q || !paged_kv_cache || !out || !mid_o || !mid_lse) {
    set_error("be_attn_run_fixed: null pointer");
    return BE_EINVAL;
  }
  int rc = check_heads(num_qo_heads, num_kv_heads, head_dim, dtype);
  if (rc) return rc;
  if (caps->max_work < 0 || caps->max_wide < 0 || caps->max_wide > caps->max_work ||
      caps->max_merge < 0 || caps->cluster < 0 || caps->cluster > 8 || page_size < 1) {
    set_error("be_attn_run_fixed: invalid caps");
    return BE_EINVAL;
  }
  if (dtype != BE_F32 && (((uintptr_t)q | (uintptr_t)paged_kv_cache) % 16 ||
                          (q_row_stride * 2) % 16)) {
    set_error("be_attn_run_fixed: q and the pool must be 16-byte aligned");
    return BE_EINVAL;
  }
  AttnParams p;
  fill_params(p, q, q_row_stride, paged_kv_cache, num_pages, page_size, num_qo_heads,
              num_kv_heads, sm_scale, out, out_row_stride, lse, mid_o, mid_lse);
  p.hdr = plan_dev;
  p.work = nullptr;
  p.qlist = nullptr;
  p.kvlist = kv_list_override;  // null: the plan's own list
  p.n_work = caps->max_work;
  p.n_wide = caps->max_wide;
  Caps c{caps->max_work, caps->max_wide, caps->max_merge, caps->cluster, true};
  c.slots = (caps->flags & BE_CAPS_SLOTS) != 0;
  return dispatch(dtype, p, nullptr, plan_dev, head_dim, c, (cudaStream_t)stream);
}

extern "C" int be_attn_run_fixed_2s(const int32_t* plan_dev, const be_attn_caps* caps, int page_size,
                                    const void* q, int64_t q_row_stride, const void* paged_kv_cache,
                                    int num_pages, int num_qo_heads, int num_kv_heads, int head_dim,
                                    int dtype, float sm_scale, void* out, int64_t out_row_stride,
                                    float* lse, float* mid_o, float* mid_lse,
                                    const int32_t* kv_list_override, void* stream, void* side_stream) {
  if (!plan_dev || !caps || !q || !paged_kv_cache || !out || !mid_o || !mid_lse) {
    set_error("be_attn_run_fixed_2s: null pointer");
    return BE_EINVAL;
  }
  int rc = check_heads(num_qo_heads, num_kv_heads, head_dim, dtype);
  if (rc) return rc;
  if (caps->max_work < 0 || caps->max_wide < 0 || caps->max_wide > caps->max_work ||
      caps->max_merge < 0 || caps->cluster < 0 || caps->cluster > 8 || page_size < 1) {
    set_error("be_attn_run_fixed_2s: invalid caps");
    return BE_EINVAL;
  }
  if (dtype != BE_F32 && (((uintptr_t)q | (uintptr_t)paged_kv_cache) % 16 ||
                          (q_row_stride * 2) % 16)) {
    set_error("be_attn_run_fixed_2s: q and the pool must be 16-byte aligned");
    return BE_EINVAL;
  }
  AttnParams p;
  fill_params(p, q, q_row_stride, paged_kv_cache, num_pages, page_size, num_qo_heads,
              num_kv_heads, sm_scale, out, out_row_stride, lse, mid_o, mid_lse);
  p.hdr = plan_dev;
  p.work = nullptr;
  p.qlist = nullptr;
  p.kvlist = kv_list_override;
  p.n_work = caps->max_work;
  p.n_wide = caps->max_wide;
  Caps c{caps->max_work, caps->max_wide, caps->max_merge, caps->cluster, true};
  c.side = (cudaStream_t)side_stream;
  c.slots = (caps->flags & BE_CAPS_SLOTS) != 0;
  return dispatch(dtype, p, nullptr, plan_dev, head_dim, c, (cudaStream_t)stream);
}
