// Persistent shared-prefix attention on tcgen05, transposed tiles (head_dim 128).
//
// A wide work item is up to 64 query-head rows (W beams x g heads of one KV
// head) against <= 128 prefix tokens.  The tile is tiny for a tensor core, so
// the cost is everything around the MMAs: getting 64 KB of K/V in, the softmax,
// and writing the rows out.  This kernel hides those behind each other:
//
//   * persistent: one CTA per SM walks a contiguous range of (item, KV head)
//     tasks with two task stages in shared memory and in TMEM, so the next
//     task's pages stream in while the current one is in softmax / epilogue,
//     and consecutive chunks of one group reuse the Q tile already in place;
//   * warp roles: warp 8 = producer (TMA for K and V pages, Q gather into the
//     swizzled layout), warp 9 = MMA issuer, warps 0-3 = softmax, warps 4-7 =
//     epilogue;
//   * transposed products keep every TMEM lane busy: S^T = K Q^T (M = 128
//     tokens, N = 64 rows) puts one token per TMEM lane, so each softmax thread
//     owns a token and its 64 scores; row maxima come from redux.sync.max.f32
//     plus a 4-warp exchange in shared memory; P^T goes to shared memory as an
//     MN-major bf16 operand; O^T = V^T P^T (M = 128 dims) puts one head dim per
//     lane, so the epilogue writes every row with coalesced stores;
//   * row sums come from the tensor core too: L = 1 P^T with an all-ones A
//     operand gives l_j in column j of every lane (the sum of the same bf16 P
//     the PV product used);
//   * the chunk is resident, so the softmax is exact and single pass.
// Every wait is bounded: on expiry the CTA records BE_EDEVICE_TIMEOUT, every
// role leaves its loop, outstanding TMA loads and MMAs are drained (bounded)
// and the TMEM is freed.
namespace be {

constexpr int WD_TOK = BE_UMMA_MAX_TOKENS;      // tokens per task (128, one per TMEM lane)
constexpr int WD_ROWS = 64;                     // query-head rows per task (MMA N)
constexpr int WD_KHALF = WD_TOK * 128;          // 64-dim half of K or V: 128 rows x 128 B
constexpr int WD_K = 2 * WD_KHALF;              // K (then P^T in its first 16 KB)
constexpr int WD_V = 2 * WD_KHALF;
constexpr int WD_Q = 2 * WD_ROWS * 128;         // Q: 2 halves x 64 rows x 128 B
constexpr int WD_STAGE = WD_K + WD_V + WD_Q;    // 80 KB
constexpr int WD_ONES = 128 * 128;              // all-ones A operand: 128 rows x 128 B (both
                                                // 64-token halves read the same block)
constexpr int WD_OUT = WD_ROWS * 128 * 4;       // output staging: 64 rows x 128 dims (fp32)
constexpr int WD_WMAX = 4 * WD_ROWS;            // per-warp row maxima (softmax scratch)
constexpr int WD_MSLOTS = 4;                    // final row maxima, one slot per task in flight
// run accumulation (consecutive chunks of one group in one CTA): running row max
// and sum [64] each, per-task rescale factors a / b [2 task parities][64] each
constexpr int WD_RUN_FLOATS = 2 * WD_ROWS + 4 * WD_ROWS;
#ifndef WD_SUSPEND_NS
#define WD_SUSPEND_NS 0
#endif
#ifndef WD_POLL_NS
#define WD_POLL_NS 32
#endif
constexpr int WD_TMEM_COLS = 512;               // S^T x2 (64 each) | (O^T | L) x2 (128 each)
constexpr uint32_t WD_S_COL = 0, WD_OL_COL = 128;
static_assert(WD_TOK == 128, "one token per TMEM lane");

constexpr size_t wd_smem_bytes() {
  return 1024 + 2 * WD_STAGE + WD_ONES + WD_OUT +
         (WD_WMAX + WD_MSLOTS * WD_ROWS + WD_ROWS + WD_RUN_FLOATS) * 4 +
         16 * 8 + 16;
}

__device__ __forceinline__ uint32_t umma_idesc_mn(int M, int N, int a_mn, int b_mn, bool bf16) {
  const uint32_t ab = bf16 ? 1u : 0u;
  return (1u << 4) | (ab << 7) | (ab << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ float warp_max(float v) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}
// tcgen05.ld of 8 / 16 consecutive columns (32 lanes x 32 bit), no wait.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// Bounded mbarrier wait by lane 0; the whole warp follows its verdict (so a
// timeout never splits the warp before a warp-collective instruction).
__device__ __forceinline__ bool wd_wait(uint64_t* b, uint32_t parity) {
#if WD_SUSPEND_NS > 0
  if (mbar_try(b, parity)) return true;
  const uint64_t t0 = gtimer();
  while (!mbar_try_sleep(b, parity, WD_SUSPEND_NS)) {
    if (gtimer() - t0 > kWaitNs) {
      atomicCAS(&g_device_status, 0, BE_EDEVICE_TIMEOUT);
      return false;
    }
  }
  return true;
#else
  return mbar_wait(b, parity);
#endif
}
__device__ __forceinline__ bool warp_wait(uint64_t* b, uint32_t parity) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = wd_wait(b, parity);
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}
__device__ __forceinline__ void named_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// Task t of the launch: KV head t / n_items, wide item t % n_items.  Each CTA
// takes a contiguous range of tasks, so its consecutive tasks are consecutive
// chunks of one group and KV head and share the Q tile.
struct WideTask {
  int item, kvh;
};
__device__ __forceinline__ WideTask wide_task(int t, int n_items) {
  return WideTask{t % n_items, t / n_items};
}

// Profiling stamps (BE_ATTN_DEBUG & 4): globaltimer per (CTA, task < 8, event < 16)
// into p.lse past the rows the merge writes.  Events: 0/1 producer start/done,
// 2/3 S / O issued, 4/5 softmax start/done, 6/7 epilogue start/done, 8/9 epilogue
// after the TMEM loads / after the row info.
__device__ __forceinline__ void wstamp(const AttnParams& p, int it, int k) {
  if ((p.debug & 4) && p.lse && it < 8)
    reinterpret_cast<unsigned long long*>(p.lse)[8192 + ((int64_t)blockIdx.x * 8 + it) * 16 + k] =
        gtimer();
}

template <typename T>
__global__ void __launch_bounds__(320, 1) attn_wide_kernel(const __grid_constant__ CUtensorMap tmap,
                                                           AttnParams p) {
  constexpr int D = 128, NH = 2;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ char smem_raw[];
  char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~uintptr_t(1023));
  char* sOnes = smem + 2 * WD_STAGE;
  char* sOut = sOnes + WD_ONES;                                         // [64 rows][128 dims]
  float* sWmax = reinterpret_cast<float*>(sOut + WD_OUT);              // [4 warps][64 rows]
  float* sM = sWmax + WD_WMAX;                                         // [4 slots][64 rows]
  float* sInv = sM + WD_MSLOTS * WD_ROWS;                              // [64] 1 / l per row
  float* sRunM = sInv + WD_ROWS;                                       // [64] running max
  float* sRunL = sRunM + WD_ROWS;                                      // [64] running sum
  float* sRunA = sRunL + WD_ROWS;                                      // [2][64] old-run scale
  float* sRunB = sRunA + 2 * WD_ROWS;                                  // [2][64] chunk scale
  uint64_t* bars = reinterpret_cast<uint64_t*>(sRunB + 2 * WD_ROWS);
  uint64_t* kq_full = bars + 0;      // [2] K pages + Q tile landed (stage)
  uint64_t* v_full = bars + 2;       // [2] V pages landed (stage)
  uint64_t* s_full = bars + 4;       // [2] S^T in TMEM
  uint64_t* p_full = bars + 6;       // [2] P^T in shared memory (128 softmax threads)
  uint64_t* o_full = bars + 8;       // [2] O^T and L in TMEM
  uint64_t* smem_empty = bars + 10;  // [2] stage's K/V/Q/P no longer read by the tensor core
  uint64_t* ol_empty = bars + 12;    // [2] epilogue has read O^T / L (128 threads)
  uint64_t* drain = bars + 14;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(bars + 15);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 15) + 1;

  resolve_plan(p);
  const int n_items = plan_n_wide(p);
  const int n_tasks = n_items * p.hkv;
  if ((int)blockIdx.x >= n_tasks) return;  // before any barrier or TMEM use
  const int grid = min((int)gridDim.x, n_tasks);
  const int t_begin = (int)((int64_t)blockIdx.x * n_tasks / grid);
  const int my_tasks = (int)((int64_t)(blockIdx.x + 1) * n_tasks / grid) - t_begin;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // all-ones operand (1.0 in bf16 / fp16); layout-free since every element is equal
  {
    const uint32_t one2 = kBf16 ? 0x3F803F80u : 0x3C003C00u;
    for (int i = tid; i < WD_ONES / 16; i += 320)
      reinterpret_cast<int4*>(sOnes)[i] = make_int4(one2, one2, one2, one2);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kq_full[s], 2);
      mbar_init(&v_full[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 128);
      mbar_init(&o_full[s], 1);
      mbar_init(&smem_empty[s], 1);
      mbar_init(&ol_empty[s], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32((const void*)tmem_slot)), "n"(WD_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int g = p.g, ps = p.page_size;

  if (warp == 8) {
    // ---------------- producer: K / V pages by TMA, Q gathered by the warp ----------------
    int issued = 0;
    int prev_q[2][3] = {{-1, -1, -1}, {-1, -1, -1}};   // (q_off, q_len, kvh) held by each stage
    for (int it = 0; it < my_tasks; ++it) {
      if (*abort_flag) break;
      const int s = it & 1;
      const WideTask tk = wide_task(t_begin + it, n_items);
      const Work w = p.work[tk.item];
      const int ntok = w.kv_end - w.kv_begin;
      if (ntok > WD_TOK || ntok <= 0 || (w.flags & BE_WORK_SLOTS) || w.q_len * g > WD_ROWS) {
        if (lane == 0) flag_range_error();   // not a plan made for this kernel
        *abort_flag = 1;
        break;
      }
      // page ids first: their latency overlaps the wait for the stage
      const int npg = (ntok + ps - 1) / ps;
      int my_page = 0;
      if (lane < npg) {
        my_page = p.kvlist[w.kv_off + w.kv_begin / ps + lane];
        if (my_page < 0 || my_page >= p.num_pages) {
          flag_range_error();
          my_page = 0;   // read page 0 instead; the status records the error
        }
      }
      if (it >= 2 && !warp_wait(&smem_empty[s], ((it >> 1) - 1) & 1)) {
        *abort_flag = 1;
        break;
      }
      if (lane == 0) wstamp(p, it, 0);
      char* sK = smem + s * WD_STAGE;
      char* sV = sK + WD_K;
      char* sQ = sV + WD_V;
      if (lane == 0) {
        mbar_expect_tx(&kq_full[s], npg * NH * TMA_BOX_BYTES);
        mbar_expect_tx(&v_full[s], npg * NH * TMA_BOX_BYTES);
      }
      for (int j = 0; j < npg; ++j) {
        const int page = __shfl_sync(0xffffffffu, my_page, j);
        if (lane == 0) {
#pragma unroll
          for (int h = 0; h < NH; ++h)
            tma_load5(smem_u32(sK + h * WD_KHALF + j * TMA_BOX_BYTES), &tmap, &kq_full[s], h * 64,
                      tk.kvh, 0, 0, page);
        }
      }
      for (int j = 0; j < npg; ++j) {
        const int page = __shfl_sync(0xffffffffu, my_page, j);
        if (lane == 0) {
#pragma unroll
          for (int h = 0; h < NH; ++h)
            tma_load5(smem_u32(sV + h * WD_KHALF + j * TMA_BOX_BYTES), &tmap, &v_full[s], h * 64,
                      tk.kvh, 0, 1, page);
        }
      }
      issued = it + 1;
      // Q tile: rows r = i * g + h (query i of the item, head kvh * g + h) in the
      // K-major 128-byte-swizzle layout [half][row][128 B].  Skipped when this
      // stage already holds the same tile (consecutive chunks of one group).
      if (!(prev_q[s][0] == w.q_off && prev_q[s][1] == w.q_len && prev_q[s][2] == tk.kvh)) {
        prev_q[s][0] = w.q_off;
        prev_q[s][1] = w.q_len;
        prev_q[s][2] = tk.kvh;
        const int rows = w.q_len * g;
        // source offset (elements) of rows lane and lane + 32; -1 = zero row
        int64_t off_a = -1, off_b = -1;
        if (lane < rows)
          off_a = (int64_t)p.qlist[w.q_off + lane / g] * p.q_row_stride +
                  (int64_t)(tk.kvh * g + lane % g) * D;
        if (lane + 32 < rows)
          off_b = (int64_t)p.qlist[w.q_off + (lane + 32) / g] * p.q_row_stride +
                  (int64_t)(tk.kvh * g + (lane + 32) % g) * D;
        const int c = lane & 15;   // 16-byte chunk of the row (8 dims)
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          int4 val[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const int r = 2 * (half * 16 + k) + (lane >> 4);   // r < 32 iff half == 0
            const int64_t oa = __shfl_sync(0xffffffffu, off_a, r & 31);
            const int64_t ob = __shfl_sync(0xffffffffu, off_b, r & 31);
            const int64_t off = half == 0 ? oa : ob;
            val[k] = off >= 0 ? *reinterpret_cast<const int4*>(reinterpret_cast<const T*>(p.q) +
                                                               off + c * 8)
                              : make_int4(0, 0, 0, 0);
          }
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const int r = 2 * (half * 16 + k) + (lane >> 4);
            *reinterpret_cast<int4*>(sQ + (c >> 3) * (WD_ROWS * 128) + r * 128 +
                                     (((c & 7) ^ (r & 7)) << 4)) = val[k];
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&kq_full[s]);
        wstamp(p, it, 1);
      }
    }
    // teardown: loads still in flight (abort only) must land before the CTA exits
    __syncwarp();
    if (lane == 0 && *abort_flag) {
      for (int it = (issued >= 2 ? issued - 2 : 0); it < issued; ++it) {
        mbar_wait(&kq_full[it & 1], (it >> 1) & 1);
        mbar_wait(&v_full[it & 1], (it >> 1) & 1);
      }
    }
  } else if (warp == 9) {
    // ---------------- MMA issuer (one lane) ----------------
    // order: S(0); then per task: S(it + 1), O(it) -- the next task's scores are
    // ready while this task's softmax finishes.  S^T buffers are free once the
    // softmax of two tasks back arrived on p_full (waited before O of that task);
    // O^T / L buffers once the epilogue of two tasks back released them.
    if (lane == 0) {
      const uint32_t id_s = umma_idesc_mn(128, WD_ROWS, 0, 0, kBf16);   // S^T = K Q^T
      const uint32_t id_o = umma_idesc_mn(128, WD_ROWS, 1, 1, kBf16);   // O^T = V^T P^T
      const uint32_t id_l = umma_idesc_mn(128, WD_ROWS, 0, 1, kBf16);   // L = 1 P^T
      auto issue_s = [&](int it) -> bool {
        const int s = it & 1;
        if (!mbar_wait(&kq_full[s], (it >> 1) & 1)) return false;
        tc_fence_after();
        const char* sK = smem + s * WD_STAGE;
        const char* sQ = sK + WD_K + WD_V;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int h = kk >> 2, koff = (kk & 3) * 32;
          const uint64_t a = umma_desc(smem_u32(sK + h * WD_KHALF) + koff, 16, 1024);
          const uint64_t b = umma_desc(smem_u32(sQ + h * (WD_ROWS * 128)) + koff, 16, 1024);
          umma_f16(tmem + WD_S_COL + s * 64, a, b, id_s, kk > 0);
        }
        umma_commit(&s_full[s]);
        wstamp(p, it, 2);
        return true;
      };
      bool ok = my_tasks > 0 ? issue_s(0) : true;
      int s_issued = my_tasks > 0 ? 1 : 0;   // S^T products issued so far
      for (int it = 0; it < my_tasks && ok; ++it) {
        const int s = it & 1;
        // O(it) needs P^T(it), V(it) and its O^T / L buffer; S(it + 1) needs K / Q of
        // the next task.  Issue whichever is ready first, S(it + 1) at the latest
        // right after O(it): neither waits behind the other's inputs.
        const uint64_t t0 = gtimer();
        for (;;) {
          if (s_issued == it + 1 && it + 1 < my_tasks &&
              mbar_try(&kq_full[(it + 1) & 1], ((it + 1) >> 1) & 1)) {
            if (!(ok = issue_s(it + 1))) break;
            ++s_issued;
          }
          if (mbar_try(&p_full[s], (it >> 1) & 1) && mbar_try(&v_full[s], (it >> 1) & 1) &&
              (it < 2 || mbar_try(&ol_empty[s], ((it >> 1) - 1) & 1)))
            break;
          __nanosleep(WD_POLL_NS);   // leave issue slots to the softmax / epilogue warps
          if (*abort_flag || gtimer() - t0 > kWaitNs) {
            if (!*abort_flag) atomicCAS(&g_device_status, 0, BE_EDEVICE_TIMEOUT);
            ok = false;
            break;
          }
        }
        if (!ok) break;
        tc_fence_after();
        const Work w = p.work[wide_task(t_begin + it, n_items).item];
        const int ksteps = ((w.kv_end - w.kv_begin + ps - 1) / ps) * ps / 16;
        const char* sP = smem + s * WD_STAGE;
        const char* sV = sP + WD_K;
        const uint32_t t_ol = tmem + WD_OL_COL + s * 128;
        for (int ks = 0; ks < ksteps; ++ks) {
          const uint64_t bp = umma_desc(smem_u32(sP + ks * 2048), 8192, 1024);
          const uint64_t av = umma_desc(smem_u32(sV + ks * 2048), WD_KHALF, 1024);
          umma_f16(t_ol, av, bp, id_o, ks > 0);
          const uint64_t a1 = umma_desc(smem_u32(sOnes) + (ks & 3) * 32, 16, 1024);
          umma_f16(t_ol + 64, a1, bp, id_l, ks > 0);
        }
        umma_commit(&o_full[s]);
        wstamp(p, it, 3);
        if (it + 2 < my_tasks) umma_commit(&smem_empty[s]);
        if (s_issued == it + 1 && it + 1 < my_tasks) {
          if (!(ok = issue_s(it + 1))) break;
          ++s_issued;
        }
      }
      if (!ok) *abort_flag = 1;
      // drain: every MMA this thread issued has completed before TMEM is freed
      umma_commit(drain);
      mbar_wait(drain, 0);
    }
    __syncwarp();
  } else if (warp < 4) {
    // ---------------- softmax: thread t owns token t of the task ----------------
    const int t = tid;
    for (int it = 0; it < my_tasks; ++it) {
      const int s = it & 1;
      const Work w = p.work[wide_task(t_begin + it, n_items).item];
      const int rows = w.q_len * g;
      const int ntok = w.kv_end - w.kv_begin;
      const int ntok_pad = ((ntok + ps - 1) / ps) * ps;
      const bool causal = (w.flags & BE_WORK_CAUSAL) != 0;
      const bool ok = !*abort_flag && warp_wait(&s_full[s], (it >> 1) & 1);
      if (!ok) *abort_flag = 1;
      if (t == 0) wstamp(p, it, 4);
      tc_fence_after();
      // Compact loops (not fully unrolled): four warp roles run different code at
      // once, so code size matters as much as instruction count here.
      const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16) + WD_S_COL + s * 64;
      // causal: row j (query j / g) sees tokens < kv_total - q_len + j / g + 1,
      // i.e. token t is visible to rows j >= (t + kv_begin - kv_total + q_len) * g
      const int jmin = causal ? max(0, w.kv_begin + t - (w.kv_total - w.q_len)) * g : 0;
      const bool tok_ok = ok && t < ntok;
      const float sc = p.scale_log2;
      float* mfin = sM + (it & (WD_MSLOTS - 1)) * WD_ROWS;
      // all 64 scores of this token in registers (one TMEM round trip)
      float x[WD_ROWS];
      {
        uint32_t u[WD_ROWS];
        if (ok) {
          tmem_ld32_nw(trow, u);
          tmem_ld32_nw(trow + 32, u + 32);
          tmem_wait();
        }
#pragma unroll
        for (int j = 0; j < WD_ROWS; ++j)
          x[j] = (tok_ok && j < rows && j >= jmin) ? __uint_as_float(u[j]) * sc : -INFINITY;
      }
      if (t == 0) wstamp(p, it, 10);
      // row maxima: warp max by redux, then across the 4 warps in shared memory
      float keep0 = -INFINITY, keep1 = -INFINITY;   // lane l keeps rows l and l + 32
#pragma unroll
      for (int j = 0; j < WD_ROWS; ++j) {
        const float m = warp_max(x[j]);
        if (j < 32) keep0 = lane == j ? m : keep0;
        else keep1 = lane == j - 32 ? m : keep1;
      }
      if (t == 0) wstamp(p, it, 11);
      sWmax[warp * WD_ROWS + lane] = keep0;
      sWmax[warp * WD_ROWS + 32 + lane] = keep1;
      named_sync(1, 128);
      if (t == 0) wstamp(p, it, 12);
      if (t < WD_ROWS)
        mfin[t] = fmaxf(fmaxf(sWmax[t], sWmax[WD_ROWS + t]),
                        fmaxf(sWmax[2 * WD_ROWS + t], sWmax[3 * WD_ROWS + t]));
      named_sync(1, 128);
      if (t == 0) wstamp(p, it, 13);
      // P^T row t = 64 values in 8 swizzled 16-byte chunks (MN-major operand)
      char* prow = smem + s * WD_STAGE + t * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float4 ma = *reinterpret_cast<const float4*>(mfin + c * 8);
        const float4 mb = *reinterpret_cast<const float4*>(mfin + c * 8 + 4);
        const float mr[8] = {ma.x, ma.y, ma.z, ma.w, mb.x, mb.y, mb.z, mb.w};
        uint32_t pk[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float e2[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float m = mr[2 * q + h] == -INFINITY ? 0.f : mr[2 * q + h];
            e2[h] = ex2(x[c * 8 + 2 * q + h] - m);   // x = -inf gives 0
          }
          pk[q] = pack2<T>(e2[0], e2[1]);
        }
        if (t < ntok_pad)
          *reinterpret_cast<int4*>(prow + ((c ^ (t & 7)) << 4)) = make_int4(pk[0], pk[1], pk[2], pk[3]);
      }
      if (t == 0) wstamp(p, it, 14);
      if (t >= ntok && t < ntok_pad) {   // last page's tail: stale V rows may be non-finite
        if (mbar_wait(&v_full[s], (it >> 1) & 1)) {
          char* vrow = smem + s * WD_STAGE + WD_K + t * 128;
#pragma unroll 1
          for (int c = 0; c < 16; ++c)
            *reinterpret_cast<int4*>(vrow + (c >> 3) * WD_KHALF + (c & 7) * 16) = make_int4(0, 0, 0, 0);
        } else {
          *abort_flag = 1;
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      mbar_arrive(&p_full[s]);
      if (t == 0) wstamp(p, it, 5);
      // Reuse of the scratch above: the warp maxima are rewritten by the next
      // task only after both named barriers of this one; final-maxima slot
      // it % 4 is rewritten by task it + 4, whose S^T product is issued after
      // O(it + 2), which waits for this task's epilogue (ol_empty).
    }
  } else {
    // ---------------- epilogue: thread d owns head dim d ----------------
    // Consecutive tasks of this CTA that are consecutive chunks of one group
    // (same KV head, queries and KV list, adjoining token ranges, both writing
    // partial rows) form a run when BE_ATTN_WIDE_RUNS is set: their O^T rows
    // accumulate in the fp32 staging rows with the exact online-softmax rescale
    // (running max M, sum L; old rows x 2^(M_old - M), chunk rows x 2^(m_c - M)),
    // and only the run's last task writes -- into the partial rows of the run's
    // first item; the other items' rows get LSE = -inf, which the merge skips.
    // A one-task run takes the per-task path below unchanged.
    const int e = warp - 4;
    const int d = e * 32 + lane;
    const bool runs_on = (p.debug & 8) != 0;
    int run_item = -1;
    auto same_run = [&](const Work& a, int ka, const Work& b, int kb) {
      return runs_on && ka == kb && a.part_base >= 0 && b.part_base >= 0 && a.q_off == b.q_off &&
             a.q_len == b.q_len && a.kv_off == b.kv_off && a.kv_end == b.kv_begin;
    };
    for (int it = 0; it < my_tasks; ++it) {
      const int s = it & 1;
      const WideTask tk = wide_task(t_begin + it, n_items);
      const Work w = p.work[tk.item];
      const int rows = w.q_len * g;
      bool first = true, last = true;
      if (runs_on) {
        if (it > 0) {
          const WideTask tp = wide_task(t_begin + it - 1, n_items);
          first = !same_run(p.work[tp.item], tp.kvh, w, tk.kvh);
        }
        if (it + 1 < my_tasks) {
          const WideTask tn = wide_task(t_begin + it + 1, n_items);
          last = !same_run(w, tk.kvh, p.work[tn.item], tn.kvh);
        }
      }
      if (first) run_item = tk.item;
      const bool ok = !*abort_flag && warp_wait(&o_full[s], (it >> 1) & 1);
      if (!ok) {
        *abort_flag = 1;
        break;
      }
      if (d == 0) wstamp(p, it, 6);
      tc_fence_after();
      const uint32_t trow = tmem + ((uint32_t)(e * 32) << 16) + WD_OL_COL + s * 128;
      // O^T row d (64 columns) and L (l_j in column j of every lane): one TMEM
      // round trip for both
      uint32_t uo[WD_ROWS];
      float l_d = 0.f;
      {
        // l_j sits in column j of every lane; thread d needs l_d only for d < 64,
        // so warps 0 and 1 each read the 32 columns of their own rows
        uint32_t ul[32];
        tmem_ld32_nw(trow, uo);
        tmem_ld32_nw(trow + 32, uo + 32);
        if (e < 2) tmem_ld32_nw(trow + 64 + e * 32, ul);
        tmem_wait();
        if (e < 2) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j == lane) l_d = __uint_as_float(ul[j]);
        }
      }
      tc_fence_before();
      mbar_arrive(&ol_empty[s]);   // TMEM no longer read: the next O / L may land
      if (d == 0) wstamp(p, it, 8);
      if (!(first && last)) {
        // ---- run accumulation (fp32 staging rows hold the run's unnormalised O) ----
        float* acc = reinterpret_cast<float*>(sOut);
        float* ra = sRunA + s * WD_ROWS;
        float* rb = sRunB + s * WD_ROWS;
        // a finished run's bulk copies must have read the staging rows
        if (first && d == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        if (d < WD_ROWS) {
          const float m_c = d < rows ? sM[(it & (WD_MSLOTS - 1)) * WD_ROWS + d] : -INFINITY;
          const float mo = first ? -INFINITY : sRunM[d];
          const float lo = first ? 0.f : sRunL[d];
          const float mn = fmaxf(mo, m_c);
          const float a = mo == -INFINITY ? 0.f : ex2(mo - mn);
          const float b = m_c == -INFINITY ? 0.f : ex2(m_c - mn);
          sRunM[d] = mn;
          sRunL[d] = lo * a + (d < rows ? l_d : 0.f) * b;
          ra[d] = a;
          rb[d] = b;
        }
        named_sync(2, 128);
#pragma unroll
        for (int j = 0; j < WD_ROWS; ++j) {   // unrolled: uo[] stays in registers
          float v = __uint_as_float(uo[j]) * rb[j];
          if (!first) v += acc[j * D + d] * ra[j];
          acc[j * D + d] = v;
        }
        if (last) {
          const Work w0 = p.work[run_item];
          if (d < rows) {
            const int i = d / g, head = tk.kvh * g + d % g;
            const float lr = sRunL[d];
            p.mid_lse[(int64_t)(w0.part_base + i) * p.hq + head] =
                lr > 0.f ? (sRunM[d] + log2f(lr)) * kLn2 : -INFINITY;
            for (int k = run_item + 1; k <= tk.item; ++k)   // the run's other partial rows
              p.mid_lse[(int64_t)(p.work[k].part_base + i) * p.hq + head] = -INFINITY;
            sInv[d] = lr > 0.f ? 1.f / lr : 0.f;
          }
          named_sync(2, 128);
#pragma unroll 8
          for (int j = 0; j < WD_ROWS; ++j) acc[j * D + d] *= sInv[j];
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          named_sync(2, 128);
          if (d == 0) {
            const uint32_t bytes = (uint32_t)(g * D * 4);
            for (int i = 0; i < w.q_len; ++i) {
              char* dst = reinterpret_cast<char*>(
                  p.mid_o + ((int64_t)(w0.part_base + i) * p.hq + (int64_t)tk.kvh * g) * D);
              asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
                           "r"(smem_u32(sOut + (size_t)i * bytes)), "r"(bytes)
                           : "memory");
            }
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          }
        }
        if (d == 0) wstamp(p, it, 7);
        continue;
      }
      // row d < rows: its LSE, and 1 / l for the rows pass
      if (d < rows) {
        const int i = d / g, head = tk.kvh * g + d % g;
        const float m_d = sM[(it & (WD_MSLOTS - 1)) * WD_ROWS + d];
        const float lse = l_d > 0.f ? (m_d + log2f(l_d)) * kLn2 : -INFINITY;
        if (w.part_base < 0) {
          if (p.lse) p.lse[(int64_t)p.qlist[w.q_off + i] * p.hq + head] = lse;
        } else {
          p.mid_lse[(int64_t)(w.part_base + i) * p.hq + head] = lse;
        }
        sInv[d] = l_d > 0.f ? 1.f / l_d : 0.f;
      }
      // the previous task's bulk stores have finished reading the staging rows
      if (d == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
      named_sync(2, 128);
      if (d == 0) wstamp(p, it, 9);
      // normalised rows -> staging [row][dim] (lanes = consecutive dims, no bank
      // conflicts); rows past `rows` hold don't-care values and are not copied
      const bool direct = w.part_base < 0;
#pragma unroll
      for (int j4 = 0; j4 < WD_ROWS; j4 += 4) {
        const float4 inv = *reinterpret_cast<const float4*>(sInv + j4);
        const float iv[4] = {inv.x, inv.y, inv.z, inv.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int j = j4 + k;
          const float v = __uint_as_float(uo[j]) * iv[k];
          if (direct)
            reinterpret_cast<T*>(sOut)[j * D + d] = from_f<T>(v);
          else
            reinterpret_cast<float*>(sOut)[j * D + d] = v;
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      named_sync(2, 128);
      // one bulk copy per query: its g heads are contiguous in the output row or
      // the partial row (g x D elements)
      if (d == 0) {
        const int esz = direct ? (int)sizeof(T) : 4;
        const uint32_t bytes = (uint32_t)(g * D * esz);
        for (int i = 0; i < w.q_len; ++i) {
          char* dst = direct ? reinterpret_cast<char*>(reinterpret_cast<T*>(p.out) +
                                                       (int64_t)p.qlist[w.q_off + i] * p.out_row_stride +
                                                       (int64_t)tk.kvh * g * D)
                             : reinterpret_cast<char*>(p.mid_o + ((int64_t)(w.part_base + i) * p.hq +
                                                                  (int64_t)tk.kvh * g) * D);
          asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
                       "r"(smem_u32(sOut + (size_t)i * bytes)), "r"(bytes)
                       : "memory");
        }
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      }
      if (d == 0) wstamp(p, it, 7);
      // row info buffer s is rewritten two tasks later, after the next task's
      // named barrier, which every thread reaches only after this loop
    }
    // the last bulk copies read the staging rows: done before the CTA's shared
    // memory can be handed to another CTA
    if (d == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(WD_TMEM_COLS) : "memory");
  }
}

static int num_sms_cached() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <typename T>
int launch_wide(const AttnParams& p, const CUtensorMap& map, int n_items, cudaStream_t st) {
  const size_t smem = wd_smem_bytes();
  static bool set = false;
  if (!set) {
    BE_CUDA_CHECK(cudaFuncSetAttribute(attn_wide_kernel<T>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    set = true;
  }
  const int tasks = n_items * p.hkv;
  const int grid = std::max(1, std::min(num_sms_cached(), tasks));
  attn_wide_kernel<T><<<grid, 320, smem, st>>>(map, p);
  BE_LAUNCH_CHECK();
  return BE_OK;
}

// BE_ATTN_WIDE=1 selects this kernel for wide tiles (head_dim 128); otherwise
// the one-task-per-CTA tcgen05 kernel runs them.  Read at every launch so a
// process can compare both.
static bool wide_enabled() {
  const char* e = getenv("BE_ATTN_WIDE");
  return e && e[0] == '1';
}

}  // namespace be
