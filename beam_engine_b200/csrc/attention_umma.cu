// Shared-prefix attention on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// One CTA = one wide work item (up to 64 query-head rows: W beams x g heads of
// one KV head over <= 128 prefix tokens, two CTAs per SM):
//   * warp 4 lane 0 streams the chunk's K and V pages with TMA (128-byte
//     swizzled boxes, K-major rows of 64 dims) and issues the MMAs;
//   * S = Q K^T: 64 x N x D as D/16 tcgen05.mma (kind::f16, M = 64, N = tokens
//     <= 128), accumulator in TMEM columns 0..N; row r sits in TMEM lane
//     32 * (r / 16) + r % 16, so every consumer warp owns 16 rows;
//   * the consumer warps read their S rows from TMEM (one lane per row),
//     do an exact single-pass softmax over the chunk (no online rescale: the
//     whole chunk is resident), write P in bf16 to shared memory in the
//     canonical K-major 128-byte-swizzle layout;
//   * O = P V: N/16 tcgen05.mma with V as an MN-major operand straight from
//     the TMA boxes, accumulator in TMEM columns 128..128+D;
//   * epilogue: O / l and the natural-log LSE to the output or a partial row.
// All mbarrier waits are bounded; on expiry the CTA flags BE_EDEVICE_TIMEOUT,
// skips the remaining MMAs, drains its copies and frees its TMEM.
namespace be {

constexpr int UM_MAX_TOK = BE_UMMA_MAX_TOKENS;   // tokens per wide work item (128)
constexpr int UM_HALF = UM_MAX_TOK * 128;         // one 64-dim half of K or V: rows x 128 B
constexpr int UM_TMEM_COLS = 2 * UM_MAX_TOK;      // S (UM_MAX_TOK cols) then O (<= 128 cols)
static_assert(UM_MAX_TOK >= 128, "O needs 128 TMEM columns after S");
constexpr int UM_KREG = 2 * UM_HALF;   // K (then P) region
constexpr int UM_VREG = 2 * UM_HALF;   // V region (D/64 halves of UM_MAX_TOK rows x 128 B)
constexpr int UM_QREG = 16 * 1024;   // Q: D/64 halves of 64 rows x 128 B (8 KB each)
constexpr size_t um_smem_bytes() { return 1024 + UM_KREG + UM_VREG + UM_QREG + 128; }

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  // SM100 shared-memory matrix descriptor: start >> 4 [0,14), LBO >> 4 [16,30),
  // SBO >> 4 [32,46), version 1 [46,48), base offset 0, layout SWIZZLE_128B (2) [61,64)
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
// Instruction descriptor, kind::f16: F32 accumulate, A/B bf16 (1) or f16 (0).
template <typename T>
__device__ __forceinline__ uint32_t umma_idesc(int M, int N, int b_mn_major) {
  const uint32_t ab = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  return (1u << 4) | (ab << 7) | (ab << 10) | ((uint32_t)b_mn_major << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// tcgen05.ld of 32 columns without the wait (batch several, then tmem_wait)
__device__ __forceinline__ void tmem_ld32_nw(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ float ex2(float x) {  // hardware base-2 exponential
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T, int D>
__global__ void __launch_bounds__(160, 2) attn_umma_kernel(const __grid_constant__ CUtensorMap tmap,
                                                        AttnParams p) {
  constexpr int NH = D / 64;
  extern __shared__ char smem_raw[];
  char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~uintptr_t(1023));
  char* sK = smem;                         // K boxes: [half][UM_MAX_TOK rows][128 B]; later P
  char* sV = sK + UM_KREG;                 // V boxes: [half][UM_MAX_TOK rows][128 B]
  char* sQ = sV + UM_VREG;                 // Q: [half][128 rows][128 B]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sQ + UM_QREG);
  uint64_t* full_k = bars + 0;
  uint64_t* full_v = bars + 1;
  uint64_t* s_done = bars + 2;
  uint64_t* o_done = bars + 3;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(bars + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 5);

  // Fixed-grid launches (p.hdr set) take a plan that is in device memory before
  // the preceding kernel starts (the step's host copy): it is read before
  // pdl_wait(), overlapping that kernel.  Otherwise, and for q and the pages
  // the preceding kernels write, everything waits.
  if (!p.hdr) pdl_wait();
  resolve_plan(p);
  if ((int)blockIdx.x >= plan_n_wide(p)) return;  // before any barrier or TMEM use
  const Work w = p.work[blockIdx.x];
  if (w.kv_end - w.kv_begin > UM_MAX_TOK || (w.flags & BE_WORK_SLOTS)) {  // not made for this kernel
    if (threadIdx.x == 0) flag_range_error();
    return;
  }
  stamp(p, 0);
  const int kvh = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = p.g, rows = w.q_len * g, ps = p.page_size;
  const int ntok = w.kv_end - w.kv_begin;                   // <= UM_MAX_TOK
  const int npg = (ntok + ps - 1) / ps;
  const int ntok_pad = npg * 16;
  const bool causal = (w.flags & BE_WORK_CAUSAL) != 0;

  if (tid == 0) {
    mbar_init(full_k, 1);
    mbar_init(full_v, 1);
    mbar_init(s_done, 1);
    mbar_init(o_done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {  // TMEM: S at columns 0..UM_MAX_TOK, O after it
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32((const void*)tmem_slot)), "n"(UM_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  stamp(p, 1);
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();

  if (warp == 4) {
    // ------------- producer: page ids (one coalesced read) -> TMA -------------
    int my_page = -1;
    if (lane < npg) my_page = p.kvlist[w.kv_off + w.kv_begin / ps + lane];
    if (lane < 16 && lane < npg && (my_page < 0 || my_page >= p.num_pages)) {
      flag_range_error();
      my_page = 0;  // read page 0 instead; the status records the error
    }
    if (lane == 0) {
      mbar_expect_tx(full_k, npg * NH * TMA_BOX_BYTES);
      mbar_expect_tx(full_v, npg * NH * TMA_BOX_BYTES);
    }
    for (int j = 0; j < npg; ++j) {
      const int page = __shfl_sync(0xffffffffu, my_page, j);
      if (lane == 0) {
#pragma unroll
        for (int h = 0; h < NH; ++h) {
          tma_load5(smem_u32(sK + h * UM_HALF + j * TMA_BOX_BYTES), &tmap, full_k, h * 64, kvh, 0, 0,
                    page);
          tma_load5(smem_u32(sV + h * UM_HALF + j * TMA_BOX_BYTES), &tmap, full_v, h * 64, kvh, 0, 1,
                    page);
        }
      }
    }
  } else {
    // ------------- consumers: Q -> smem in the K-major SW128 layout -------------
    for (int idx = tid; idx < 64 * (D / 8); idx += 128) {
      const int r = idx / (D / 8), c = idx % (D / 8);
      int4 val = make_int4(0, 0, 0, 0);
      if (r < rows) {
        const int qi = p.qlist[w.q_off + r / g];
        val = *reinterpret_cast<const int4*>(reinterpret_cast<const T*>(p.q) + qi * p.q_row_stride +
                                             (int64_t)(kvh * g + r % g) * D + c * 8);
      }
      *reinterpret_cast<int4*>(sQ + (c >> 3) * 8192 + r * 128 + (((c & 7) ^ (r & 7)) << 4)) = val;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();

  // ------------- S = Q K^T  (M = 64: row r lives in TMEM lane 32*(r/16) + r%16) -------------
  if (warp == 4 && lane == 0) {
    if (!mbar_wait(full_k, 0)) {
      *abort_flag = 1;
      mbar_arrive(s_done);
    } else {
      tc_fence_after();
      const uint32_t idesc = umma_idesc<T>(64, ntok_pad, 0);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int h = kk >> 2, koff = (kk & 3) * 32;
        const uint64_t a = umma_desc(smem_u32(sQ + h * 8192) + koff, 16, 1024);
        const uint64_t b = umma_desc(smem_u32(sK + h * UM_HALF) + koff, 16, 1024);
        umma_f16(tmem, a, b, idesc, kk > 0);
      }
      umma_commit(s_done);
    }
  }
  // ------------- softmax: lanes 0-15 of each warp own one row each, P -> smem -------------
  float m_row = -INFINITY, l_row = 0.f;
  const int r = warp * 16 + lane;     // meaningful for lane < 16
  const bool row_lane = lane < 16 && r < rows;
  if (warp < 4) {
    const bool ok = mbar_wait(s_done, 0) && !*abort_flag;
    stamp(p, 6);
    tc_fence_after();
    if (!ok) *abort_flag = 1;
    if (ok && warp * 16 < rows) {  // whole warps: tcgen05.ld is warp-collective
      const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
      int lim = w.kv_end;
      if (causal && row_lane) lim = min(w.kv_end, w.kv_total - w.q_len + r / g + 1);
      const int tlim = row_lane ? lim - w.kv_begin : 0;  // valid tokens of this row
      float mx = -INFINITY;
      for (int c0 = 0; c0 < ntok_pad; c0 += 64) {
        uint32_t v[64];
        tmem_ld32_nw(trow + c0, v);
        if (c0 + 32 < ntok_pad) tmem_ld32_nw(trow + c0 + 32, v + 32);
        tmem_wait();
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (c0 + i < tlim) mx = fmaxf(mx, __uint_as_float(v[i]));
      }
      mx *= p.scale_log2;        // scale > 0: max commutes with the scaling
      m_row = mx;
      stamp(p, 2);
      float sum = 0.f;
      for (int c0 = 0; c0 < ntok_pad; c0 += 64) {
        uint32_t v[64];
        tmem_ld32_nw(trow + c0, v);
        if (c0 + 32 < ntok_pad) tmem_ld32_nw(trow + c0 + 32, v + 32);
        tmem_wait();
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 64; i += 2) {
          const float e0 = (c0 + i < tlim) ? ex2(__uint_as_float(v[i]) * p.scale_log2 - mx) : 0.f;
          const float e1 =
              (c0 + i + 1 < tlim) ? ex2(__uint_as_float(v[i + 1]) * p.scale_log2 - mx) : 0.f;
          sum += e0 + e1;
          pk[i / 2] = pack2<T>(e0, e1);
        }
        if (lane < 16) {  // P row r, tokens c0..c0+63 = one 64-token block, 8 swizzled chunks
          char* prow = sK + (c0 >> 6) * 8192 + r * 128;
          const int nch = min(8, (ntok_pad - c0) >> 3);
#pragma unroll
          for (int q8 = 0; q8 < 8; ++q8)
            if (q8 < nch)
              *reinterpret_cast<int4*>(prow + ((q8 ^ (r & 7)) << 4)) =
                  make_int4(pk[q8 * 4], pk[q8 * 4 + 1], pk[q8 * 4 + 2], pk[q8 * 4 + 3]);
        }
      }
      l_row = sum;
    }
    // zero V rows past the chunk in the last page (stale pool data may be non-finite)
    if (ok && ntok < ntok_pad) {
      if (mbar_wait(full_v, 0)) {
        for (int idx = tid; idx < (ntok_pad - ntok) * NH * 8; idx += 128) {
          const int rr = ntok + idx / (NH * 8), rest = idx % (NH * 8);
          *reinterpret_cast<int4*>(sV + (rest >> 3) * UM_HALF + rr * 128 + (rest & 7) * 16) =
              make_int4(0, 0, 0, 0);
        }
      } else {
        *abort_flag = 1;
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  stamp(p, 3);
  tc_fence_after();

  // ------------- O = P V -------------
  if (warp == 4 && lane == 0) {
    if (*abort_flag || !mbar_wait(full_v, 0)) {
      *abort_flag = 1;
      mbar_arrive(o_done);
    } else {
      const uint32_t idesc = umma_idesc<T>(64, D, 1);
      for (int ks = 0; ks < ntok_pad / 16; ++ks) {
        const uint64_t a = umma_desc(smem_u32(sK + (ks >> 2) * 8192) + (ks & 3) * 32, 16, 1024);
        const uint64_t b = umma_desc(smem_u32(sV + ks * 2048), UM_HALF, 1024);
        umma_f16(tmem + UM_MAX_TOK, a, b, idesc, ks > 0);
      }
      umma_commit(o_done);
    }
  }
  // ------------- epilogue -------------
  if (warp < 4) {
    const bool ok = mbar_wait(o_done, 0) && !*abort_flag;
    stamp(p, 7);
    tc_fence_after();
    if (ok && warp * 16 < rows) {
      const uint32_t trow = tmem + UM_MAX_TOK + ((uint32_t)(warp * 32) << 16);
      const float inv = l_row > 0.f ? 1.f / l_row : 0.f;
      const int i = r / g, head = kvh * g + r % g;
      for (int c0 = 0; c0 < D; c0 += 64) {
        uint32_t u[64];
        tmem_ld32_nw(trow + c0, u);
        tmem_ld32_nw(trow + c0 + 32, u + 32);
        tmem_wait();
        if (!row_lane) continue;
        float v[64];
#pragma unroll
        for (int k = 0; k < 64; ++k) v[k] = __uint_as_float(u[k]) * inv;
        if (w.part_base < 0) {
          const int qi = p.qlist[w.q_off + i];
          T* dst = reinterpret_cast<T*>(p.out) + qi * p.out_row_stride + (int64_t)head * D + c0;
#pragma unroll
          for (int k = 0; k < 64; k += 8) {
            uint32_t pk[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) pk[q] = pack2<T>(v[k + 2 * q], v[k + 2 * q + 1]);
            *reinterpret_cast<int4*>(dst + k) = make_int4(pk[0], pk[1], pk[2], pk[3]);
          }
        } else {
          float* dst = p.mid_o + ((int64_t)(w.part_base + i) * p.hq + head) * D + c0;
#pragma unroll
          for (int k = 0; k < 64; k += 4)
            *reinterpret_cast<float4*>(dst + k) = make_float4(v[k], v[k + 1], v[k + 2], v[k + 3]);
        }
      }
      if (row_lane) {
        const float lse = l_row > 0.f ? (m_row + log2f(l_row)) * kLn2 : -INFINITY;
        if (w.part_base < 0) {
          if (p.lse) p.lse[(int64_t)p.qlist[w.q_off + i] * p.hq + head] = lse;
        } else {
          p.mid_lse[(int64_t)(w.part_base + i) * p.hq + head] = lse;
        }
      }
    }
  }
  stamp(p, 4);
  // ------------- teardown: copies landed, TMEM freed -------------
  if (tid == 0 && *abort_flag) {
    mbar_wait(full_k, 0);
    mbar_wait(full_v, 0);
  }
  tc_fence_before();
  __syncthreads();
  stamp(p, 5);
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(UM_TMEM_COLS) : "memory");
  }
}

template <typename T, int D>
int launch_umma(const AttnParams& p, const CUtensorMap& map, int n_items, cudaStream_t st) {
  const size_t smem = um_smem_bytes();
  static bool set = false;
  if (!set) {
    BE_CUDA_CHECK(cudaFuncSetAttribute(attn_umma_kernel<T, D>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    set = true;
  }
  BE_CUDA_CHECK(launch_pdl(attn_umma_kernel<T, D>, dim3(n_items, p.hkv), 160, smem, st, map, p));
  return BE_OK;
}

// BE_ATTN_UMMA=0 in the environment keeps wide tiles on the mma.sync kernel (A/B runs).
static bool umma_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("BE_ATTN_UMMA");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

}  // namespace be
