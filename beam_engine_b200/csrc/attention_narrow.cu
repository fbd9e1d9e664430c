// Narrow-tile paged attention with every KV head in one CTA (sm_100a).
//
// A narrow work item is one beam's suffix (q_len * g <= 16 query-head rows per
// KV head).  Giving each (item, head) its own CTA makes Hkv times more CTAs than
// SMs, each too short to hide its start-up latency; here one CTA takes the item
// for all heads:
//   * warp Hkv (producer, one lane) streams page after page: per page and head,
//     K and V boxes of 16 tokens x 64 dims (128-byte swizzle) by TMA into a
//     3-page ring, one mbarrier per page with complete_tx;
//   * warp h (h < Hkv) owns KV head h: its g query heads x q_len queries in the
//     16 rows of one m16n8k16 tile, S = Q K^T and O += P V on the tensor cores
//     with an online softmax in registers, then writes its rows (output or
//     partial row + natural-log LSE) straight from registers -- no cross-warp
//     reduction at all.
// Waits are bounded (BE_EDEVICE_TIMEOUT on expiry, then drain).
namespace be {

constexpr int NR_NS = 3;   // pages in flight per CTA (each page = all heads)

template <int D>
constexpr int nr_head_stage() { return 2 * (D / 64) * TMA_BOX_BYTES; }   // K+V, one head
template <int D>
constexpr size_t nr_smem_bytes(int hkv) {
  return 1024 + (size_t)NR_NS * hkv * nr_head_stage<D>() + (size_t)hkv * 16 * D * 2 + 2 * NR_NS * 8 + 16;
}

template <typename T, int D>
__global__ void __launch_bounds__(288) attn_narrow_kernel(const __grid_constant__ CUtensorMap tmap,
                                                          AttnParams p, int w0) {
  constexpr int KSTEPS = D / 16;
  constexpr int HS = nr_head_stage<D>();
  extern __shared__ char smem_raw[];
  char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~uintptr_t(1023));
  resolve_plan(p);
  const int wi = (w0 < 0 ? plan_n_wide(p) : w0) + blockIdx.x;
  if (wi >= plan_n_work(p)) return;
  const Work w = p.work[wi];
  if (w.flags & BE_WORK_SLOTS) {
    if (threadIdx.x == 0) flag_range_error();
    return;
  }
  const int hkv = p.hkv;
  const int STAGE = hkv * HS;
  char* sStage = smem;                                   // [NR_NS][hkv][K|V][half][16][128 B]
  char* sQ = smem + NR_NS * STAGE;                       // [hkv][16][D]
  uint64_t* full = reinterpret_cast<uint64_t*>(sQ + hkv * 16 * D * 2);
  uint64_t* empty = full + NR_NS;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + NR_NS);
  volatile int* issued_ptr = abort_flag + 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = p.g, rows = w.q_len * g, ps = p.page_size;
  const bool causal = (w.flags & BE_WORK_CAUSAL) != 0;
  const int npg = (w.kv_end - w.kv_begin + ps - 1) / ps;
  const int first_page = w.kv_begin / ps;
  if (tid == 0) {
    for (int s = 0; s < NR_NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], hkv);
    }
    *abort_flag = 0;
    *issued_ptr = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == hkv) {
    // ---------------- producer ----------------
    const uint32_t tx = STAGE;
    bool stop = false;
    int j = 0;
    for (int base = 0; base < npg && !stop; base += 32) {
      const int jj = base + lane;
      const int my_page = jj < npg ? p.kvlist[w.kv_off + first_page + jj] : -1;
      const int cnt = min(32, npg - base);
      for (int k = 0; k < cnt; ++k) {
        const int page = __shfl_sync(0xffffffffu, my_page, k);
        j = base + k;
        int go = 1;
        if (lane == 0) {
          const int s = j % NR_NS;
          if (j >= NR_NS && !mbar_wait(&empty[s], ((j / NR_NS) - 1) & 1)) {
            *abort_flag = 1;
            go = 0;
          } else if (*abort_flag) {
            go = 0;
          } else if (page < 0 || page >= p.num_pages) {
            flag_range_error();
            mbar_arrive(&full[s]);
          } else {
            mbar_expect_tx(&full[s], tx);
            const uint32_t dst = smem_u32(sStage + s * STAGE);
            for (int h = 0; h < hkv; ++h)
#pragma unroll
              for (int pl = 0; pl < 2; ++pl)
#pragma unroll
                for (int hf = 0; hf < D / 64; ++hf)
                  tma_load5(dst + h * HS + (pl * (D / 64) + hf) * TMA_BOX_BYTES, &tmap, &full[s],
                            hf * 64, h, 0, pl, page);
          }
        }
        go = __shfl_sync(0xffffffffu, go, 0);
        if (!go) {
          stop = true;
          break;
        }
        ++j;
      }
    }
    if (lane == 0) *issued_ptr = stop ? j : npg;
  } else if (warp < hkv) {
    // ---------------- consumer: KV head `warp` ----------------
    const int kvh = warp;
    char* myQ = sQ + kvh * 16 * D * 2;
    for (int idx = lane; idx < 16 * (D / 8); idx += 32) {
      const int r = idx / (D / 8), c = idx % (D / 8);
      int4 val = make_int4(0, 0, 0, 0);
      if (r < rows) {
        const int qi = p.qlist[w.q_off + r / g];
        val = *reinterpret_cast<const int4*>(reinterpret_cast<const T*>(p.q) + qi * p.q_row_stride +
                                             (int64_t)(kvh * g + r % g) * D + c * 8);
      }
      *reinterpret_cast<int4*>(myQ + swz<D>(r, c)) = val;
    }
    __syncwarp();
    uint32_t qf[KSTEPS][4];
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk)
      ldsm_x4(smem_u32(myQ + swz<D>(lane % 16, kk * 2 + (lane / 16))), qf[kk][0], qf[kk][1],
              qf[kk][2], qf[kk][3]);
    const int r0 = lane / 4, r1 = r0 + 8;
    int lim0 = w.kv_end, lim1 = w.kv_end;
    if (causal) {
      if (r0 < rows) lim0 = min(w.kv_end, w.kv_total - w.q_len + r0 / g + 1);
      if (r1 < rows) lim1 = min(w.kv_end, w.kv_total - w.q_len + r1 / g + 1);
    }
    float o[D / 8][4];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    for (int j = 0; j < npg; ++j) {
      const int s = j % NR_NS;
      if (*abort_flag || !mbar_wait(&full[s], (j / NR_NS) & 1)) {
        *abort_flag = 1;
        break;
      }
      char* st = sStage + s * STAGE + kvh * HS;
      const int t0 = w.kv_begin + j * ps;
      const int valid = min(ps, w.kv_end - t0);
      if (valid < 16) {
        for (int idx = lane; idx < (16 - valid) * (D / 8); idx += 32) {
          const int r = valid + idx / (D / 8), c = idx % (D / 8);
          *reinterpret_cast<int4*>(st + stage_off<D>(1, r, c)) = make_int4(0, 0, 0, 0);
        }
        __syncwarp();
      }
      float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk) {
        const int mi = lane / 8;
        const int tok = ((mi >> 1) << 3) + (lane % 8);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(smem_u32(st + stage_off<D>(0, tok, kk * 2 + (mi & 1))), b0, b1, b2, b3);
        mma16816<T>(sc[0], qf[kk], b0, b1);
        mma16816<T>(sc[1], qf[kk], b2, b3);
      }
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int t = t0 + n * 8 + 2 * (lane % 4) + (c & 1);
          const float x = t < (c < 2 ? lim0 : lim1) ? sc[n][c] * p.scale_log2 : -INFINITY;
          sc[n][c] = x;
          if (c < 2) mx0 = fmaxf(mx0, x); else mx1 = fmaxf(mx1, x);
        }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float a0 = (mn0 == -INFINITY) ? 1.f : exp2f(m0 - mn0);
      const float a1 = (mn1 == -INFINITY) ? 1.f : exp2f(m1 - mn1);
      float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
      for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float mref = c < 2 ? mn0 : mn1;
          const float e = (mref == -INFINITY) ? 0.f : exp2f(sc[n][c] - mref);
          sc[n][c] = e;
          if (c < 2) ps0 += e; else ps1 += e;
        }
      l0 = l0 * a0 + ps0;
      l1 = l1 * a1 + ps1;
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        o[i][0] *= a0; o[i][1] *= a0; o[i][2] *= a1; o[i][3] *= a1;
      }
      const uint32_t pa4[4] = {pack2<T>(sc[0][0], sc[0][1]), pack2<T>(sc[0][2], sc[0][3]),
                               pack2<T>(sc[1][0], sc[1][1]), pack2<T>(sc[1][2], sc[1][3])};
#pragma unroll
      for (int dn = 0; dn < D / 16; ++dn) {
        const int mi = lane / 8;
        const int tok = ((mi & 1) << 3) + (lane % 8);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(smem_u32(st + stage_off<D>(1, tok, dn * 2 + (mi >> 1))), b0, b1, b2, b3);
        mma16816<T>(o[2 * dn], pa4, b0, b1);
        mma16816<T>(o[2 * dn + 1], pa4, b2, b3);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    // rows r0 / r1 of this head, straight from registers
    const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = half ? r1 : r0;
      if (r >= rows) continue;
      const float inv = half ? inv1 : inv0;
      const int i = r / g, head = kvh * g + r % g;
      if (w.part_base < 0) {
        const int qi = p.qlist[w.q_off + i];
        T* dst = reinterpret_cast<T*>(p.out) + qi * p.out_row_stride + (int64_t)head * D;
#pragma unroll
        for (int k = 0; k < D / 8; ++k) {
          const int d = k * 8 + 2 * (lane % 4);
          *reinterpret_cast<uint32_t*>(dst + d) =
              pack2<T>(o[k][half * 2] * inv, o[k][half * 2 + 1] * inv);
        }
      } else {
        float* dst = p.mid_o + ((int64_t)(w.part_base + i) * p.hq + head) * D;
#pragma unroll
        for (int k = 0; k < D / 8; ++k) {
          const int d = k * 8 + 2 * (lane % 4);
          *reinterpret_cast<float2*>(dst + d) =
              make_float2(o[k][half * 2] * inv, o[k][half * 2 + 1] * inv);
        }
      }
      if (lane % 4 == 0) {
        const float m = half ? m1 : m0, l = half ? l1 : l0;
        const float lse = l > 0.f ? (m + log2f(l)) * kLn2 : -INFINITY;
        if (w.part_base < 0) {
          if (p.lse) p.lse[(int64_t)p.qlist[w.q_off + i] * p.hq + head] = lse;
        } else {
          p.mid_lse[(int64_t)(w.part_base + i) * p.hq + head] = lse;
        }
      }
    }
  }
  // drain after an abort: every issued TMA lands before the CTA leaves
  __syncthreads();
  if (tid == 0 && *abort_flag) {
    const int issued = *issued_ptr;
    for (int s = 0; s < NR_NS && s < issued; ++s) {
      const int last = s + ((issued - 1 - s) / NR_NS) * NR_NS;
      mbar_wait(&full[s], (last / NR_NS) & 1);
    }
  }
}

template <typename T, int D>
int launch_narrow(const AttnParams& p, const CUtensorMap& map, int w0, int n_items,
                  cudaStream_t st) {
  const size_t smem = nr_smem_bytes<D>(p.hkv);
  static bool set = false;
  if (!set) {
    BE_CUDA_CHECK(cudaFuncSetAttribute(attn_narrow_kernel<T, D>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)nr_smem_bytes<D>(8)));
    set = true;
  }
  attn_narrow_kernel<T, D><<<n_items, 32 * (p.hkv + 1), smem, st>>>(map, p, w0);
  BE_LAUNCH_CHECK();
  return BE_OK;
}

static bool narrow_enabled() {  // BE_ATTN_NARROW=0 keeps narrow tiles on the per-head kernel
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("BE_ATTN_NARROW");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

}  // namespace be
