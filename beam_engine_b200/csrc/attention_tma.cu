// Paged decode attention, TMA-fed (sm_100a): the bf16/fp16 fast path of be_attn_run.
//
// Layout: one CTA = 4 consumer warps + 1 producer warp; a thread-block cluster
// of `cs` CTAs shares one work item x KV head and splits its pages.
//   * producer (one elected lane): per page, 2 x (D/64) TMA box loads of 2 KB
//     (K|V x 64-dim halves, 16 tokens each, 128-byte swizzle) from a 5-D tensor
//     map over the pool [pages][2][page_size][kv_heads][dims] into an 8-stage
//     ring, each stage signalled by an mbarrier with complete_tx;
//   * consumers: S = Q K^T and O += P V on the tensor cores (mma.sync
//     m16n8k16, fp32 accumulate), online softmax in registers, several pages
//     per step for instruction-level parallelism; wide tiles (<= 64 rows)
//     give each warp 16 rows and every 4-page step, narrow tiles (<= 16 rows)
//     give each warp every 4th 2-page step;
//   * end: the CTA folds its warps' (m, l, O) in shared memory, then rank 0 of
//     the cluster folds the peers' states over distributed shared memory (no
//     HBM traffic for the split); the result goes to the output or to a
//     partial row for the LSE merge.
// Every mbarrier wait is bounded (globaltimer, 2 s): on expiry the CTA records
// BE_EDEVICE_TIMEOUT in the device status word, drains and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <unordered_map>

namespace be {

constexpr int TMA_NS = 8;                   // pages in flight per CTA
constexpr int TMA_BOX_BYTES = 16 * 64 * 2;  // 16 tokens x 64 dims x 2 B
constexpr uint64_t kWaitNs = 2000000000ull;

__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* b, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait with a suspend-time hint: the thread sleeps in hardware until the
// phase completes or about `ns` nanoseconds pass (no issue slots burnt spinning).
__device__ __forceinline__ bool mbar_try_sleep(uint64_t* b, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}
// Bounded wait; false (and the device status set) on timeout.  The clock is
// read once every 256 polls: %globaltimer reads are slow and a warp that spins
// on them steals issue slots from the warps doing the work.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity) {
  if (mbar_try(b, parity)) return true;
  uint64_t t0 = 0;
  for (uint32_t n = 1;; ++n) {
    if (mbar_try(b, parity)) return true;
    if ((n & 255) == 0) {
      const uint64_t t = gtimer();
      if (t0 == 0) {
        t0 = t;
      } else if (t - t0 > kWaitNs) {
        atomicCAS(&g_device_status, 0, BE_EDEVICE_TIMEOUT);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void tma_load5(uint32_t dst, const CUtensorMap* map, uint64_t* bar,
                                          int c0, int c1, int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(dst),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ uint32_t map_peer(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_peer(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// Byte offset of (token row r, 16-byte dim chunk c) inside one page stage:
// [plane][dim half][16 rows][128 B], chunk XOR (row & 7) = TMA 128-byte swizzle.
template <int D>
__device__ __forceinline__ uint32_t stage_off(int plane, int r, int c) {
  return (plane * (D / 64) + (c >> 3)) * TMA_BOX_BYTES + r * 128 + (((c & 7) ^ (r & 7)) << 4);
}

template <int D>
constexpr int tma_stage_bytes() { return 2 * (D / 64) * TMA_BOX_BYTES; }
template <int D>
constexpr size_t tma_smem_bytes() {
  return 1024 + TMA_NS * tma_stage_bytes<D>() + 64 * D * 2 + 2 * TMA_NS * 8 + 16;
}
// fold buffers (4 slots x 16 rows or 1 slot x 64 rows, m/l, per-rank weights)
// reuse the stage ring
static_assert(64 * 132 * 4 + 2 * 64 * 4 + 64 * 8 * 4 <= TMA_NS * 2 * 2 * TMA_BOX_BYTES,
              "fold buffers must fit in the stage ring (D = 128)");
static_assert(64 * 68 * 4 + 2 * 64 * 4 + 64 * 8 * 4 <= TMA_NS * 2 * 1 * TMA_BOX_BYTES,
              "fold buffers must fit in the stage ring (D = 64)");

// Profiling stamps (BE_ATTN_DEBUG & 4): globaltimer per phase into p.lse.
__device__ __forceinline__ void stamp(const AttnParams& p, int phase) {
  if ((p.debug & 4) && p.lse && threadIdx.x == 0)
    reinterpret_cast<unsigned long long*>(p.lse)[((int64_t)blockIdx.x * gridDim.y + blockIdx.y) * 8 +
                                                 phase] = gtimer();
}

template <typename T, int D, int MT>
__device__ void tma_tile(const CUtensorMap* tmap, const AttnParams& p, const Work& w, int kvh,
                         int cs, int rank, char* smem) {
  constexpr int NWM = MT / 16, NWK = 4 / NWM, KSTEPS = D / 16;
  // pages per consumer step: wide tiles take 4 (all warps share each step),
  // narrow tiles 2 (each warp owns every 4th step, 4 steps fill the ring)
  constexpr int PG = MT == 64 ? 4 : 2;
  static_assert(TMA_NS % (PG * NWK) == 0 || NWK == 1, "ring must hold one step per warp");
  constexpr int STAGE = tma_stage_bytes<D>();
  char* sStage = smem;                                   // TMA_NS * STAGE, 1024-aligned
  char* sQ = smem + TMA_NS * STAGE;                      // [64][D] T
  uint64_t* full = reinterpret_cast<uint64_t*>(sQ + 64 * D * 2);
  uint64_t* empty = full + TMA_NS;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + TMA_NS);
  volatile int* issued_ptr = abort_flag + 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = p.g, rows = w.q_len * g, ps = p.page_size;
  const bool causal = (w.flags & BE_WORK_CAUSAL) != 0;
  const int n_pages = (w.kv_end - w.kv_begin + ps - 1) / ps;
  const int pa = (int)((int64_t)n_pages * rank / cs);
  const int pb = (int)((int64_t)n_pages * (rank + 1) / cs);
  const int npg = pb - pa;
  const int first_page = w.kv_begin / ps + pa;
  stamp(p, 0);
  if (tid == 0) {
    for (int s = 0; s < TMA_NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], MT == 64 ? 4 : 1);
    }
    *abort_flag = 0;
    *issued_ptr = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();   // barriers ready: the producer starts streaming now
  if (warp < 4) {    // Q tile (overlaps the first TMA loads), zero rows past q_len * g
    constexpr int CPR = D / 8;
    constexpr int PER = MT * CPR / 128;
    int4 val[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int idx = tid + k * 128;
      const int r = idx / CPR, c = idx % CPR;
      val[k] = make_int4(0, 0, 0, 0);
      if (r < rows) {
        const int qi = p.qlist[w.q_off + r / g];
        val[k] = *reinterpret_cast<const int4*>(reinterpret_cast<const T*>(p.q) +
                                                qi * p.q_row_stride + (int64_t)(kvh * g + r % g) * D +
                                                c * 8);
      }
    }
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int idx = tid + k * 128;
      *reinterpret_cast<int4*>(sQ + swz<D>(idx / CPR, idx % CPR)) = val[k];
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");  // consumer warps only
  }
  stamp(p, 1);

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int warp_m = warp % NWM, warp_k = warp / NWM;
  const int r0 = warp_m * 16 + lane / 4, r1 = r0 + 8;

  if (warp == 4) {
    // ---------------- producer ----------------
    // Page ids are fetched 32 at a time by the whole warp (one coalesced load)
    // and handed to lane 0 by shuffles, so the issue loop never waits on a
    // dependent global load.
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
          const int s = j % TMA_NS;
          if (j >= TMA_NS && !mbar_wait(&empty[s], ((j / TMA_NS) - 1) & 1)) {
            *abort_flag = 1;
            go = 0;
          } else if (*abort_flag) {
            go = 0;
          } else if (page < 0 || page >= p.num_pages) {
            flag_range_error();
            mbar_arrive(&full[s]);  // consumers see stale data; the status records the error
          } else {
            mbar_expect_tx(&full[s], tx);
            const uint32_t dst = smem_u32(sStage + s * STAGE);
#pragma unroll
            for (int pl = 0; pl < 2; ++pl)
#pragma unroll
              for (int h = 0; h < D / 64; ++h)
                tma_load5(dst + (pl * (D / 64) + h) * TMA_BOX_BYTES, tmap, &full[s], h * 64, kvh,
                          0, pl, page);
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
  } else {
    // ---------------- consumers ----------------
    uint32_t qf[KSTEPS][4];
    {
      const int r = warp_m * 16 + (lane % 16);
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk)
        ldsm_x4(smem_u32(sQ + swz<D>(r, kk * 2 + (lane / 16))), qf[kk][0], qf[kk][1], qf[kk][2],
                qf[kk][3]);
    }
    int lim0 = w.kv_end, lim1 = w.kv_end;
    if (causal) {
      if (r0 < rows) lim0 = min(w.kv_end, w.kv_total - w.q_len + r0 / g + 1);
      if (r1 < rows) lim1 = min(w.kv_end, w.kv_total - w.q_len + r1 / g + 1);
    }
    // Each step takes PG consecutive pages (16*PG tokens): PG*2 independent
    // n-tiles per k-step for S, one softmax pass, PG k-steps per d-tile for PV.
    const int ngroups = (npg + PG - 1) / PG;
    for (int gi = warp_k; gi < ngroups; gi += NWK) {
      const int j0 = gi * PG;
      bool ok = !*abort_flag;
#pragma unroll
      for (int pi = 0; pi < PG; ++pi) {
        const int j = j0 + pi;
        if (ok && j < npg && !mbar_wait(&full[j % TMA_NS], (j / TMA_NS) & 1)) ok = false;
      }
      if (!ok) {
        *abort_flag = 1;
        break;
      }
      if (gi == warp_k) stamp(p, 2);
      if (p.debug & 1) {
        __syncwarp();
        if (lane == 0)
          for (int pi = 0; pi < PG; ++pi)
            if (j0 + pi < npg) mbar_arrive(&empty[(j0 + pi) % TMA_NS]);
        continue;
      }
      float sc[2 * PG][4];
#pragma unroll
      for (int n = 0; n < 2 * PG; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
      for (int pi = 0; pi < PG; ++pi) {
        const int j = j0 + pi;
        if (j >= npg) break;
        char* st = sStage + (j % TMA_NS) * STAGE;
        const int valid = min(ps, w.kv_end - (w.kv_begin + (pa + j) * ps));
        if (valid < 16) {  // zero V rows past the range (stale pool data may be non-finite)
          for (int idx = lane; idx < (16 - valid) * (D / 8); idx += 32) {
            const int r = valid + idx / (D / 8), c = idx % (D / 8);
            *reinterpret_cast<int4*>(st + stage_off<D>(1, r, c)) = make_int4(0, 0, 0, 0);
          }
        }
      }
      __syncwarp();
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk) {
#pragma unroll
        for (int pi = 0; pi < PG; ++pi) {
          const int j = j0 + pi;
          if (j < npg) {
            const char* st = sStage + (j % TMA_NS) * STAGE;
            const int mi = lane / 8;
            const int tok = ((mi >> 1) << 3) + (lane % 8);
            uint32_t b0, b1, b2, b3;
            ldsm_x4(smem_u32(st + stage_off<D>(0, tok, kk * 2 + (mi & 1))), b0, b1, b2, b3);
            mma16816<T>(sc[2 * pi], qf[kk], b0, b1);
            mma16816<T>(sc[2 * pi + 1], qf[kk], b2, b3);
          }
        }
      }
      const int tbase = w.kv_begin + (pa + j0) * ps;
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int n = 0; n < 2 * PG; ++n)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int t = tbase + n * 8 + 2 * (lane % 4) + (c & 1);
          const bool in = (j0 + n / 2) < npg && t < (c < 2 ? lim0 : lim1);
          const float x = in ? sc[n][c] * p.scale_log2 : -INFINITY;
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
      for (int n = 0; n < 2 * PG; ++n)
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
#pragma unroll
      for (int pi = 0; pi < PG; ++pi) {
        const int j = j0 + pi;
        if (j >= npg) break;
        const char* st = sStage + (j % TMA_NS) * STAGE;
        uint32_t pa4[4] = {pack2<T>(sc[2 * pi][0], sc[2 * pi][1]),
                           pack2<T>(sc[2 * pi][2], sc[2 * pi][3]),
                           pack2<T>(sc[2 * pi + 1][0], sc[2 * pi + 1][1]),
                           pack2<T>(sc[2 * pi + 1][2], sc[2 * pi + 1][3])};
#pragma unroll
        for (int dn = 0; dn < D / 16; ++dn) {
          const int mi = lane / 8;
          const int tok = ((mi & 1) << 3) + (lane % 8);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(smem_u32(st + stage_off<D>(1, tok, dn * 2 + (mi >> 1))), b0, b1, b2, b3);
          mma16816<T>(o[2 * dn], pa4, b0, b1);
          mma16816<T>(o[2 * dn + 1], pa4, b2, b3);
        }
      }
      __syncwarp();
      if (lane == 0) {
#pragma unroll
        for (int pi = 0; pi < PG; ++pi)
          if (j0 + pi < npg) mbar_arrive(&empty[(j0 + pi) % TMA_NS]);
      }
    }
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    stamp(p, 3);
  }
  // Drain: after an abort, wait (bounded) for every issued TMA before the ring
  // memory is reused; normally every issued page was consumed already.
  __syncthreads();
  if (tid == 0 && *abort_flag) {
    const int issued = *issued_ptr;
    for (int s = 0; s < TMA_NS && s < issued; ++s) {
      const int last = s + ((issued - 1 - s) / TMA_NS) * TMA_NS;  // last use of stage s
      mbar_wait(&full[s], (last / TMA_NS) & 1);
    }
  }
  __syncthreads();

  stamp(p, 4);
  if (p.debug & 2) return;
  // ---- fold the warps' states: slot k holds the rows of warp column k ----
  // (row pitch D + 4 floats keeps the fragment stores free of bank conflicts)
  constexpr int OS = D + 4;
  float* sO = reinterpret_cast<float*>(sStage);          // [NWK][MT][OS]
  float* sM = sO + NWK * MT * OS;                        // [NWK][MT]
  float* sL = sM + NWK * MT;
  float* sW = sL + NWK * MT;                             // [MT][8] fold weights
  if (warp < 4) {
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      const int d = i * 8 + 2 * (lane % 4);
      *reinterpret_cast<float2*>(&sO[(warp_k * MT + r0) * OS + d]) = make_float2(o[i][0], o[i][1]);
      *reinterpret_cast<float2*>(&sO[(warp_k * MT + r1) * OS + d]) = make_float2(o[i][2], o[i][3]);
    }
    if (lane % 4 == 0) {
      sM[warp_k * MT + r0] = m0; sL[warp_k * MT + r0] = l0;
      sM[warp_k * MT + r1] = m1; sL[warp_k * MT + r1] = l1;
    }
  }
  __syncthreads();
  const int nthr = blockDim.x;
  if (NWK > 1) {  // fold slots into slot 0 with per-row weights computed once
    if (tid < MT) {
      float mt = -INFINITY, lt = 0.f;
      for (int k = 0; k < NWK; ++k) mt = fmaxf(mt, sM[k * MT + tid]);
      for (int k = 0; k < NWK; ++k) {
        const float wk = mt == -INFINITY ? 0.f : exp2f(sM[k * MT + tid] - mt);
        sW[tid * 8 + k] = wk;
        lt += wk * sL[k * MT + tid];
      }
      sW[tid * 8 + 4] = mt;
      sW[tid * 8 + 5] = lt;
    }
    __syncthreads();
    for (int idx = tid; idx < MT * (D / 4); idx += nthr) {
      const int r = idx / (D / 4), d = (idx % (D / 4)) * 4;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int k = 0; k < NWK; ++k) {
        const float4 v = *reinterpret_cast<const float4*>(&sO[(k * MT + r) * OS + d]);
        const float wk = sW[r * 8 + k];
        acc.x += wk * v.x; acc.y += wk * v.y; acc.z += wk * v.z; acc.w += wk * v.w;
      }
      *reinterpret_cast<float4*>(&sO[r * OS + d]) = acc;
    }
    __syncthreads();
    if (tid < MT) {
      sM[tid] = sW[tid * 8 + 4];
      sL[tid] = sW[tid * 8 + 5];
    }
    __syncthreads();
  }
  stamp(p, 5);
  // ---- fold the cluster's CTAs: rank 0 reads the peers over DSMEM ----
  if (cs > 1) cluster_sync();
  if (rank == 0) {
    const uint32_t aO = smem_u32(sO), aM = smem_u32(sM), aL = smem_u32(sL);
    if (tid < rows) {  // per-row weight of each rank, normalised by the folded sum
      const int r = tid;
      float mc[8], lc[8];
      float mt = -INFINITY;
      for (int c = 0; c < cs; ++c) {
        mc[c] = c ? ld_peer(map_peer(aM + r * 4, c)) : sM[r];
        lc[c] = c ? ld_peer(map_peer(aL + r * 4, c)) : sL[r];
        mt = fmaxf(mt, mc[c]);
      }
      float lt = 0.f;
      for (int c = 0; c < cs; ++c) lt += (mt == -INFINITY ? 0.f : exp2f(mc[c] - mt)) * lc[c];
      for (int c = 0; c < cs; ++c)
        sW[r * 8 + c] = (lt > 0.f && mt != -INFINITY) ? exp2f(mc[c] - mt) / lt : 0.f;
      const int i = r / g, head = kvh * g + r % g;
      const float lse = lt > 0.f ? (mt + log2f(lt)) * kLn2 : -INFINITY;
      if (w.part_base < 0) {
        if (p.lse) p.lse[(int64_t)p.qlist[w.q_off + i] * p.hq + head] = lse;
      } else {
        p.mid_lse[(int64_t)(w.part_base + i) * p.hq + head] = lse;
      }
    }
    __syncthreads();
    for (int idx = tid; idx < rows * (D / 4); idx += nthr) {
      const int r = idx / (D / 4), d = (idx % (D / 4)) * 4;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int c = 0; c < cs; ++c) {
        float4 v;
        if (c == 0) {
          v = *reinterpret_cast<const float4*>(&sO[r * OS + d]);
        } else {
          const uint32_t a = map_peer(aO + (r * OS + d) * 4, c);
          asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
                       : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                       : "r"(a)
                       : "memory");
        }
        const float wc = sW[r * 8 + c];
        acc.x += wc * v.x; acc.y += wc * v.y; acc.z += wc * v.z; acc.w += wc * v.w;
      }
      const int i = r / g, head = kvh * g + r % g;
      if (w.part_base < 0) {
        const int qi = p.qlist[w.q_off + i];
        T* dst = reinterpret_cast<T*>(p.out) + qi * p.out_row_stride + (int64_t)head * D + d;
        dst[0] = from_f<T>(acc.x); dst[1] = from_f<T>(acc.y);
        dst[2] = from_f<T>(acc.z); dst[3] = from_f<T>(acc.w);
      } else {
        *reinterpret_cast<float4*>(p.mid_o + ((int64_t)(w.part_base + i) * p.hq + head) * D + d) =
            acc;
      }
    }
  }
  if (cs > 1) cluster_sync();  // peers keep their shared memory until rank 0 is done
  stamp(p, 6);
}

template <typename T, int D>
__global__ void __launch_bounds__(160) attn_tma_kernel(const __grid_constant__ CUtensorMap tmap,
                                                       AttnParams p, int cs, int w0) {
  extern __shared__ char smem_raw[];
  char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~uintptr_t(1023));
  resolve_plan(p);
  // w0 < 0: the wide items ran on the tensor-core kernel; skip them (count from the plan)
  const int wi = (w0 < 0 ? plan_n_wide(p) : w0) + blockIdx.x / cs;
  if (wi >= plan_n_work(p)) return;  // whole clusters leave together (same wi)
  const int rank = cs > 1 ? (int)cluster_rank() : 0;
  const Work w = p.work[wi];
  if (w.flags & BE_WORK_SLOTS) {     // slot lists are not page lists: not for this kernel
    if (threadIdx.x == 0) flag_range_error();
    return;
  }
  if (wi < plan_n_wide(p))
    tma_tile<T, D, 64>(&tmap, p, w, blockIdx.y, cs, rank, smem);
  else
    tma_tile<T, D, 16>(&tmap, p, w, blockIdx.y, cs, rank, smem);
}

// ---- host: tensor maps over one layer's pool, cached by address ----
struct MapKey {
  const void* base;
  int pages, ps, hkv, d, dtype;
  bool operator==(const MapKey& o) const {
    return base == o.base && pages == o.pages && ps == o.ps && hkv == o.hkv && d == o.d &&
           dtype == o.dtype;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.base) ^ ((size_t)k.pages << 7) ^ ((size_t)k.hkv << 29);
  }
};

static int get_pool_map(const void* pool, int pages, int ps, int hkv, int d, int dtype,
                        CUtensorMap* out) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  std::lock_guard<std::mutex> lk(mu);
  MapKey key{pool, pages, ps, hkv, d, dtype};
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
  const int elt = 2;
  cuuint64_t dims[5] = {(cuuint64_t)d, (cuuint64_t)hkv, (cuuint64_t)ps, 2, (cuuint64_t)pages};
  cuuint64_t strides[4] = {(cuuint64_t)d * elt, (cuuint64_t)hkv * d * elt,
                           (cuuint64_t)ps * hkv * d * elt, (cuuint64_t)2 * ps * hkv * d * elt};
  cuuint32_t box[5] = {64, 1, (cuuint32_t)ps, 1, 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUtensorMap m;
  CUresult r = encode(&m,
                      dtype == BE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                      5, const_cast<void*>(pool), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return BE_ECUDA;
  }
  if (cache.size() > 4096) cache.clear();
  cache[key] = m;
  *out = m;
  return BE_OK;
}

// BE_ATTN_CP_ASYNC=1 in the environment selects the cp.async kernel (A/B runs).
static bool force_cp_async() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("BE_ATTN_CP_ASYNC");
    v = (e && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

// Cluster size: split the heaviest work item so that its per-CTA share is no
// more than the average per-CTA page count with two resident CTAs per SM.
// BE_ATTN_CLUSTER=<n> forces n (1..8).
static int pick_cluster(const be_attn_plan_info* info, int hkv, int ps) {
  const char* e = getenv("BE_ATTN_CLUSTER");
  if (e && atoi(e) >= 1 && atoi(e) <= 8) return atoi(e);
  const int max_item_pages = (info->max_item_tokens + ps - 1) / ps;
  const int64_t total_pages = ((int64_t)info->total_tokens + ps - 1) / ps;
  const int64_t slots = 148 * 2;
  const int64_t avg = std::max<int64_t>(8, (total_pages * hkv + slots - 1) / slots);
  int cs = (int)((max_item_pages + avg - 1) / avg);
  if (cs < 1) cs = 1;
  if (cs > 8) cs = 8;
  while (cs > 1 && (int64_t)info->n_work * cs > (1 << 30)) cs >>= 1;
  return cs;
}

template <typename T, int D>
int launch_tma(const AttnParams& p, const CUtensorMap& map, int cs, int w0, int n_items,
               cudaStream_t st) {
  const size_t smem = tma_smem_bytes<D>();
  static bool set = false;
  if (!set) {
    BE_CUDA_CHECK(cudaFuncSetAttribute(attn_tma_kernel<T, D>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_items * cs, p.hkv, 1);
  cfg.blockDim = dim3(160, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  BE_CUDA_CHECK(cudaLaunchKernelEx(&cfg, attn_tma_kernel<T, D>, map, p, cs, w0));
  return BE_OK;
}

}  // namespace be
