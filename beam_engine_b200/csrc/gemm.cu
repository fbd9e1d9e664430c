// Weight-streaming GEMM for the decode step: Y[T][N] = X[T][K] * W[N][K]^T with
// T <= 128 rows (the beams of a step), bf16 in, fp32 accumulate, bf16 or fp32 out.
//
// In decode every projection is a skinny GEMM that reads its weight matrix once
// per step, so it is HBM-bound on W.  The library GEMM splits these shapes into
// too few CTAs for small N (O and down projections: 32 output tiles of 128 on
// 148 SMs) and reaches 2.5-4.9 TB/s.  Here:
//   * the MMA is transposed: Y^T tile (128 output features x T tokens) =
//     W tile (M = 128, K-major) x X^T (N = T, K-major), accumulated in TMEM
//     (128 lanes x T fp32 columns), one tcgen05.mma per 16-wide K step;
//   * a CTA owns one 128-feature tile and a K range (split-K): the grid is sized
//     to one wave of one CTA per SM; W and X tiles (64 K-elements, 128-byte
//     swizzle) stream by TMA through a 6-stage ring (192 KB in flight per SM:
//     a CTA's bandwidth is bytes in flight / latency);
//   * one elected lane issues TMA, one elected lane issues the MMAs, then all
//     four warps drain TMEM (warp w holds features 32w..32w+31) and write Y;
//   * split-K runs as a thread-block cluster along the K splits: each CTA parks
//     its fp32 partial tile in its own shared memory, and after a cluster
//     barrier CTA r sums token rows r/S.. of all S partials over distributed
//     shared memory and writes them -- no partials in HBM, no second kernel.
// Every wait is bounded (BE_EDEVICE_TIMEOUT, then drain and free the TMEM).
namespace be {

constexpr int GM_BM = 128;                 // output features per tile (MMA M)
constexpr int GM_BN = 128;                 // tokens (MMA N), T <= 128
constexpr int GM_BK = 64;                  // K elements per stage (one 128-byte swizzle row)
constexpr int GM_ST = 6;                   // pipeline stages (192 KB: one CTA per SM)
constexpr int GM_A = GM_BM * GM_BK * 2;    // 16 KB
constexpr int GM_B = GM_BN * GM_BK * 2;    // 16 KB
constexpr size_t gm_smem_bytes() { return 1024 + GM_ST * (GM_A + GM_B) + (2 * GM_ST + 2) * 8 + 16; }

__device__ __forceinline__ void tma_load2(uint32_t dst, const CUtensorMap* map, uint64_t* bar,
                                          int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

template <typename OutT>
__global__ void __launch_bounds__(128) gemm_tn_kernel(const __grid_constant__ CUtensorMap map_w,
                                                      const __grid_constant__ CUtensorMap map_x,
                                                      OutT* __restrict__ y, int64_t ldy,
                                                      int T, int N, int K, int kb_per_split,
                                                      int x_rows) {
  extern __shared__ char smem_raw[];
  char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + GM_ST * (GM_A + GM_B));
  uint64_t* empty = full + GM_ST;
  uint64_t* done = empty + GM_ST;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(done + 1) + 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m0 = blockIdx.x * GM_BM;
  const int split = blockIdx.y;
  const int kb_total = K / GM_BK;
  const int kb0 = split * kb_per_split;
  const int kb1 = min(kb_total, kb0 + kb_per_split);
  const int nkb = kb1 - kb0;
  if (tid == 0) {
    for (int s = 0; s < GM_ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32((const void*)tmem_slot)), "n"(GM_BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---- producer: W tile rows m0.., X rows 0..127 (rows >= T / >= N read as zeros) ----
    for (int i = 0; i < nkb; ++i) {
      const int s = i % GM_ST;
      if (i >= GM_ST && !mbar_wait(&empty[s], ((i / GM_ST) - 1) & 1)) {
        *abort_flag = 1;
        break;
      }
      char* sa = smem + s * (GM_A + GM_B);
      mbar_expect_tx(&full[s], GM_A + x_rows * 128);
      tma_load2(smem_u32(sa), &map_w, &full[s], (kb0 + i) * GM_BK, m0);
      tma_load2(smem_u32(sa + GM_A), &map_x, &full[s], (kb0 + i) * GM_BK, 0);
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(GM_BN >> 3) << 17) |
                           ((uint32_t)(GM_BM >> 4) << 24);   // f32 acc, bf16 A/B, K-major both
    int i = 0;
    for (; i < nkb; ++i) {
      const int s = i % GM_ST;
      if (*abort_flag || !mbar_wait(&full[s], (i / GM_ST) & 1)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const char* sa = smem + s * (GM_A + GM_B);
#pragma unroll
      for (int kk = 0; kk < GM_BK / 16; ++kk) {
        const uint64_t a = umma_desc(smem_u32(sa) + kk * 32, 16, 1024);
        const uint64_t b = umma_desc(smem_u32(sa + GM_A) + kk * 32, 16, 1024);
        umma_f16(tmem, a, b, idesc, (i > 0 || kk > 0) ? 1u : 0u);
      }
      umma_commit(&empty[s]);
    }
    umma_commit(done);   // every MMA issued above has completed when this arrives
  }
  __syncwarp();
  // ---- epilogue: warp w owns features m0 + 32 w + lane; columns are tokens ----
  const bool ok = mbar_wait(done, 0) && !*abort_flag;
  tc_fence_after();
  const int f = m0 + warp * 32 + lane;
  const int S = gridDim.y;   // CTAs of the cluster = K splits
  const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
  if (S == 1) {
    if (ok) {
      for (int c0 = 0; c0 < T; c0 += 32) {   // T is uniform: whole warps load together
        uint32_t v[32];
        tmem_ld32_nw(trow + c0, v);
        tmem_wait();
        if (f < N) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (c0 + j < T) y[(int64_t)(c0 + j) * ldy + f] = from_f<OutT>(__uint_as_float(v[j]));
        }
      }
    }
  } else {
    // partial tile -> own shared memory [token][128 features] (the stage ring is idle now)
    float* part = reinterpret_cast<float*>(smem);
    for (int c0 = 0; c0 < T; c0 += 32) {
      uint32_t v[32];
      if (ok) {
        tmem_ld32_nw(trow + c0, v);
        tmem_wait();
      }
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (c0 + j < T) part[(c0 + j) * GM_BM + warp * 32 + lane] = ok ? __uint_as_float(v[j]) : 0.f;
    }
    cluster_sync();   // every partial is in place (release / acquire across the cluster)
    // CTA rank r sums token rows [r*T/S, (r+1)*T/S) of all partials, 4 features per thread
    const uint32_t rank = cluster_rank();
    const int t0 = (int)((int64_t)rank * T / S), t1 = (int)((int64_t)(rank + 1) * T / S);
    const uint32_t base = smem_u32(part);
    const int n_e = (t1 - t0) * (GM_BM / 4);
    // four float4 groups per thread per round, every peer's load issued before
    // any sum, so the distributed-shared-memory latency is paid once per round
    for (int e0 = tid; e0 < n_e; e0 += 4 * 128) {
      float4 acc[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int q = 0; q < S; ++q) {
        float4 b[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int e = e0 + u * 128;
          b[u] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (e < n_e) {
            const int t = t0 + e / (GM_BM / 4), f4 = (e % (GM_BM / 4)) * 4;
            const uint32_t pa = map_peer(base + (uint32_t)((t * GM_BM + f4) * 4), (uint32_t)q);
            asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
                         : "=f"(b[u].x), "=f"(b[u].y), "=f"(b[u].z), "=f"(b[u].w)
                         : "r"(pa)
                         : "memory");
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          acc[u].x += b[u].x;
          acc[u].y += b[u].y;
          acc[u].z += b[u].z;
          acc[u].w += b[u].w;
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int e = e0 + u * 128;
        if (e >= n_e) continue;
        const int t = t0 + e / (GM_BM / 4), fg = m0 + (e % (GM_BM / 4)) * 4;
        OutT* dst = y + (int64_t)t * ldy + fg;
        if (fg + 0 < N) dst[0] = from_f<OutT>(acc[u].x);
        if (fg + 1 < N) dst[1] = from_f<OutT>(acc[u].y);
        if (fg + 2 < N) dst[2] = from_f<OutT>(acc[u].z);
        if (fg + 3 < N) dst[3] = from_f<OutT>(acc[u].w);
      }
    }
    cluster_sync();   // no CTA leaves while a peer may still read its partials
  }
  // ---- teardown: on abort, loads still in flight land before the CTA exits ----
  if (tid == 0 && *abort_flag) {
    for (int i = max(0, nkb - GM_ST); i < nkb; ++i) mbar_wait(&full[i % GM_ST], (i / GM_ST) & 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(GM_BN)
                 : "memory");
  }
}

struct Map2Key {
  const void* p;
  int64_t rows, cols, ld;
  int box;
  bool operator==(const Map2Key& o) const {
    return p == o.p && rows == o.rows && cols == o.cols && ld == o.ld && box == o.box;
  }
};
struct Map2Hash {
  size_t operator()(const Map2Key& k) const {
    return std::hash<const void*>()(k.p) ^ (std::hash<int64_t>()(k.rows) * 31) ^
           (std::hash<int64_t>()(k.cols) * 131) ^ (std::hash<int64_t>()(k.ld) * 1031);
  }
};

// bf16 2-D tensor map [rows][cols] (row stride ld elements), box 64 cols x box_rows
// rows, 128-byte swizzle; cached by (pointer, shape, box).
static int get_map2(const void* p, int64_t rows, int64_t cols, int64_t ld, int box_rows,
                    CUtensorMap* out) {
  static std::mutex mu;
  static std::unordered_map<Map2Key, CUtensorMap, Map2Hash> cache;
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  std::lock_guard<std::mutex> lk(mu);
  Map2Key key{p, rows, cols, ld, box_rows};
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return BE_OK;
  }
  if (!encode) {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
            cudaSuccess ||
        !fn) {
      set_error("cuTensorMapEncodeTiled unavailable");
      return BE_ECUDA;
    }
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)GM_BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMap m;
  CUresult r = encode(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(p), dims, strides,
                      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (gemm) failed (%d)", (int)r);
    return BE_ECUDA;
  }
  if (cache.size() > 4096) cache.clear();
  cache[key] = m;
  *out = m;
  return BE_OK;
}

template <typename OutT>
static int launch_gemm(const CUtensorMap& mw, const CUtensorMap& mx, void* y, int64_t ldy, int T,
                       int N, int K, int splits, int kb_per_split, int x_rows, cudaStream_t st) {
  static bool set = false;
  if (!set) {
    BE_CUDA_CHECK(cudaFuncSetAttribute(gemm_tn_kernel<OutT>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)gm_smem_bytes()));
    set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((N + GM_BM - 1) / GM_BM, splits, 1);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.dynamicSmemBytes = gm_smem_bytes();
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = splits;   // the K splits of one tile form a cluster
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  BE_CUDA_CHECK(cudaLaunchKernelEx(&cfg, gemm_tn_kernel<OutT>, mw, mx, reinterpret_cast<OutT*>(y),
                                   ldy, T, N, K, kb_per_split, x_rows));
  return BE_OK;
}

}  // namespace be

using namespace be;

extern "C" int be_gemm_tn(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y,
                          int64_t ldy, int T, int N, int K, int out_dtype, int split_k,
                          float* workspace, int64_t workspace_floats, void* stream) {
  if (!x || !w || !y || T < 1 || T > GM_BN || N < GM_BM || K < GM_BK || K % GM_BK ||
      (out_dtype != BE_BF16 && out_dtype != BE_F32) || ldx < K || ldw < K || ldy < N ||
      ldx % 8 || ldw % 8 || ((uintptr_t)x | (uintptr_t)w) % 16) {
    set_error("be_gemm_tn: unsupported shape (T %d <= %d, N %d, K %d %% %d, ld %lld/%lld/%lld, "
              "16-byte aligned operands)", T, GM_BN, N, K, GM_BK, (long long)ldx, (long long)ldw,
              (long long)ldy);
    return BE_EINVAL;
  }
  const int tiles = (N + GM_BM - 1) / GM_BM;
  const int kb = K / GM_BK;
  // split-K = cluster size: the largest power of two <= 8 that keeps the grid
  // within one wave (one CTA per SM) with at least 4 K blocks per split
  int splits = split_k;
  if (splits <= 0) {
    const int sms = num_sms_cached();
    splits = 1;
    while (splits < 8 && tiles * splits * 2 <= sms && kb / (splits * 2) >= 4) splits *= 2;
  }
  if (splits != 1 && splits != 2 && splits != 4 && splits != 8) {
    set_error("be_gemm_tn: split_k %d must be 1, 2, 4 or 8", splits);
    return BE_EINVAL;
  }
  const int per = (kb + splits - 1) / splits;
  if ((int64_t)per * (splits - 1) >= kb) {
    set_error("be_gemm_tn: split_k %d leaves an empty K range (K %d)", splits, K);
    return BE_EINVAL;
  }
  (void)workspace;
  (void)workspace_floats;
  // X rows per tile: T rounded up to 8 (rows past T in the box read as zeros;
  // MMA columns past the box only feed output columns that are never stored)
  const int x_rows = std::min(GM_BN, (T + 7) / 8 * 8);
  CUtensorMap mw, mx;
  int rc = get_map2(w, N, K, ldw, GM_BM, &mw);
  if (rc != BE_OK) return rc;
  rc = get_map2(x, T, K, ldx, x_rows, &mx);
  if (rc != BE_OK) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  return out_dtype == BE_BF16
             ? launch_gemm<__nv_bfloat16>(mw, mx, y, ldy, T, N, K, splits, per, x_rows, st)
             : launch_gemm<float>(mw, mx, y, ldy, T, N, K, splits, per, x_rows, st);
}
