// Paged decode attention over a work-item plan, plus the LSE merge.
//
// One CTA = one work item x one KV head.  A work item is "q_len queries of one
// group against tokens [kv_begin, kv_end) of that group's paged KV sequence";
// with group size g = Hq/Hkv its rows are q_len*g query-head pairs that all
// read the same K/V rows, so the tile is a small dense contraction:
//
//   * wide tiles (up to 64 rows: the shared prefix of W beams)   4 warps x 16 rows
//   * narrow tiles (up to 16 rows: one beam's suffix, g heads)    4 warps split the KV
//
// K/V tiles of 64 tokens stream HBM -> shared memory with 16-byte cp.async
// (zero-filled past the range, XOR-swizzled rows), double buffered; S = Q K^T
// and O += P V run on the tensor cores (mma.sync m16n8k16, fp32 accumulate)
// with the online softmax in registers (quad shuffles, base-2 exponent).
// Results are either written straight to the output (single-partial queries)
// or stored as fp32 partial (o, lse) rows that merge_kernel combines.
//
// The fp32 storage path (parity mode) runs a CUDA-core kernel with the same
// plan format: a warp per row, lanes across head_dim, warp-shuffle dot products.
#include "common.cuh"

namespace be {

struct Work {
  int q_off, q_len, kv_off, kv_begin, kv_end, kv_total, part_base, flags;
};
static_assert(sizeof(Work) == sizeof(be_attn_work), "work layout");

struct AttnParams {
  const Work* work;
  const int32_t* qlist;
  const int32_t* kvlist;
  const char* q;
  int64_t q_row_stride;  // elements
  const char* pool;
  int num_pages, page_size, hq, hkv, g;
  float scale_log2;      // sm_scale * log2(e)
  char* out;
  int64_t out_row_stride;
  float* lse;
  float* mid_o;
  float* mid_lse;
  int n_work, n_wide;
  int debug;             // BE_ATTN_DEBUG switches; bit 3 = BE_ATTN_WIDE_RUNS
  const int32_t* hdr;    // plan header on the device (fixed-grid launches), else null
};

// Work / wide-item counts: from the launch when the grid was sized to the
// plan, from the plan header on the device for fixed (capturable) grids.
__device__ __forceinline__ int plan_n_work(const AttnParams& p) { return p.hdr ? p.hdr[0] : p.n_work; }
__device__ __forceinline__ int plan_n_wide(const AttnParams& p) { return p.hdr ? p.hdr[1] : p.n_wide; }
// Fixed-grid launches pass only the plan base: list pointers come from the
// header offsets (a kv list override, if any, is already in p.kvlist).
__device__ __forceinline__ void resolve_plan(AttnParams& p) {
  if (p.hdr) {
    p.work = reinterpret_cast<const Work*>(p.hdr + p.hdr[5]);
    p.qlist = p.hdr + p.hdr[6];
    if (!p.kvlist) p.kvlist = p.hdr + p.hdr[7];
  }
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr int KT = 64;  // KV tokens per shared-memory tile

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(sz));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& a, uint32_t& b, uint32_t& c,
                                        uint32_t& d) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& a, uint32_t& b, uint32_t& c,
                                          uint32_t& d) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
               : "r"(addr));
}

template <typename T>
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float* c, const uint32_t* a, uint32_t b0,
                                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float* c, const uint32_t* a, uint32_t b0,
                                                 uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Row address of token t of a work item (K plane; V is +page_size*hkv*D).
__device__ __forceinline__ int64_t token_row(const AttnParams& p, const Work& w, int t, int kvh,
                                             int D, bool& ok) {
  int page, slot;
  if (w.flags & BE_WORK_SLOTS) {
    const int s = p.kvlist[w.kv_off + t];
    page = s / p.page_size;
    slot = s - page * p.page_size;
  } else {
    page = p.kvlist[w.kv_off + t / p.page_size];
    slot = t % p.page_size;
  }
  ok = page >= 0 && page < p.num_pages && slot >= 0;
  if (!ok) return 0;
  return ((((int64_t)page * 2) * p.page_size + slot) * p.hkv + kvh) * D;
}

// Swizzled byte offset of (row, 16-byte chunk) in a [rows][D] tile.
template <int D>
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return row * (D * 2) + ((chunk ^ (row & 7)) << 4);
}

template <typename T, int D>
__device__ __forceinline__ void load_kv_tile(const AttnParams& p, const Work& w, int kvh, int t0,
                                             char* sK, char* sV) {
  constexpr int CPR = D / 8;           // 16-byte chunks per row
  constexpr int RPI = 128 / CPR;       // rows covered per pass
  const int tid = threadIdx.x;
  const int c = tid % CPR;
  const int64_t vofs = (int64_t)p.page_size * p.hkv * D;
#pragma unroll
  for (int k = 0; k < KT / RPI; ++k) {
    const int r = tid / CPR + k * RPI;
    const int t = t0 + r;
    bool ok = t < w.kv_end;
    int64_t row = 0;
    if (ok) {
      row = token_row(p, w, t, kvh, D, ok);
      if (!ok) flag_range_error();
    }
    const T* base = reinterpret_cast<const T*>(p.pool) + row + c * 8;
    cp_async16(smem_u32(sK + swz<D>(r, c)), base, ok);
    cp_async16(smem_u32(sV + swz<D>(r, c)), base + vofs, ok);
  }
}

// One wide (MT = 64) or narrow (MT = 16) tile.
template <typename T, int D, int MT>
__device__ void attn_tile(const AttnParams& p, const Work& w, int kvh, char* smem) {
  constexpr int NWM = MT / 16;         // warps along rows
  constexpr int NWK = 4 / NWM;         // warps along KV
  constexpr int KSTEPS = D / 16;
  constexpr int TILE_BYTES = KT * D * 2;
  char* sQ = smem;                                  // [64][D]
  char* sKV = smem + 64 * D * 2;                    // 2 stages x (K, V)
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int warp_m = warp % NWM, warp_k = warp / NWM;
  const int g = p.g;
  const int rows = w.q_len * g;
  const bool causal = (w.flags & BE_WORK_CAUSAL) != 0;

  // ---- Q tile -> smem (zero rows past q_len*g) ----
  {
    constexpr int CPR = D / 8;
    for (int idx = tid; idx < MT * CPR; idx += 128) {
      const int r = idx / CPR, c = idx % CPR;
      int4 val = make_int4(0, 0, 0, 0);
      if (r < rows) {
        const int i = r / g, j = r % g;
        const int qi = p.qlist[w.q_off + i];
        const T* src = reinterpret_cast<const T*>(p.q) + qi * p.q_row_stride +
                       (int64_t)(kvh * g + j) * D + c * 8;
        val = *reinterpret_cast<const int4*>(src);
      }
      *reinterpret_cast<int4*>(sQ + swz<D>(r, c)) = val;
    }
  }
  const int t_begin = w.kv_begin, t_end = w.kv_end;
  const int n_tiles = (t_end - t_begin + KT - 1) / KT;
  if (n_tiles > 0) {
    load_kv_tile<T, D>(p, w, kvh, t_begin, sKV, sKV + TILE_BYTES);
  }
  cp_commit();
  __syncthreads();

  // Q fragments for this warp's 16 rows.
  uint32_t qf[KSTEPS][4];
  {
    const int r = warp_m * 16 + (lane % 16);
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
      const int chunk = kk * 2 + (lane / 16);
      ldsm_x4(smem_u32(sQ + swz<D>(r, chunk)), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
    }
  }

  // Per-thread rows r0 = lane/4, r1 = r0 + 8 (within this warp's 16).
  const int r0 = warp_m * 16 + lane / 4, r1 = r0 + 8;
  int lim0 = t_end, lim1 = t_end;
  if (causal) {
    if (r0 < rows) lim0 = min(t_end, w.kv_total - w.q_len + r0 / g + 1);
    if (r1 < rows) lim1 = min(t_end, w.kv_total - w.q_len + r1 / g + 1);
  }
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  for (int it = 0; it < n_tiles; ++it) {
    const int t0 = t_begin + it * KT;
    if (it + 1 < n_tiles) {
      char* nb = sKV + ((it + 1) & 1) * 2 * TILE_BYTES;
      load_kv_tile<T, D>(p, w, kvh, t0 + KT, nb, nb + TILE_BYTES);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const char* sK = sKV + (it & 1) * 2 * TILE_BYTES;
    const char* sV = sK + TILE_BYTES;
#pragma unroll
    for (int st = warp_k; st < KT / 16; st += NWK) {
      const int tb = st * 16;
      if (t0 + tb >= t_end) break;
      float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk) {
        const int m = lane / 8;
        const int tok = tb + ((m >> 1) << 3) + (lane % 8);
        const int chunk = kk * 2 + (m & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(smem_u32(sK + swz<D>(tok, chunk)), b0, b1, b2, b3);
        mma16816<T>(s[0], qf[kk], b0, b1);
        mma16816<T>(s[1], qf[kk], b2, b3);
      }
      // mask + online softmax (base 2)
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int n = 0; n < 2; ++n) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int t = t0 + tb + n * 8 + 2 * (lane % 4) + (c & 1);
          const int lim = c < 2 ? lim0 : lim1;
          const float x = t < lim ? s[n][c] * p.scale_log2 : -INFINITY;
          s[n][c] = x;
          if (c < 2) mx0 = fmaxf(mx0, x); else mx1 = fmaxf(mx1, x);
        }
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
      for (int n = 0; n < 2; ++n) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float mref = c < 2 ? mn0 : mn1;
          const float e = (mref == -INFINITY) ? 0.f : exp2f(s[n][c] - mref);
          s[n][c] = e;
          if (c < 2) ps0 += e; else ps1 += e;
        }
      }
      l0 = l0 * a0 + ps0;
      l1 = l1 * a1 + ps1;
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        o[i][0] *= a0; o[i][1] *= a0; o[i][2] *= a1; o[i][3] *= a1;
      }
      uint32_t pa[4];
      pa[0] = pack2<T>(s[0][0], s[0][1]);
      pa[1] = pack2<T>(s[0][2], s[0][3]);
      pa[2] = pack2<T>(s[1][0], s[1][1]);
      pa[3] = pack2<T>(s[1][2], s[1][3]);
#pragma unroll
      for (int dn = 0; dn < D / 16; ++dn) {
        const int m = lane / 8;
        const int tok = tb + ((m & 1) << 3) + (lane % 8);
        const int chunk = dn * 2 + (m >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(smem_u32(sV + swz<D>(tok, chunk)), b0, b1, b2, b3);
        mma16816<T>(o[2 * dn], pa, b0, b1);
        mma16816<T>(o[2 * dn + 1], pa, b2, b3);
      }
    }
    __syncthreads();
  }
  // full row sums across the quad
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

  auto emit = [&](int r, int d, float v0, float v1) {  // two consecutive columns
    if (r >= rows) return;
    const int i = r / g, j = r % g;
    const int head = kvh * g + j;
    if (w.part_base < 0) {
      const int qi = p.qlist[w.q_off + i];
      T* dst = reinterpret_cast<T*>(p.out) + qi * p.out_row_stride + (int64_t)head * D + d;
      dst[0] = from_f<T>(v0);
      dst[1] = from_f<T>(v1);
    } else {
      float* dst = p.mid_o + ((int64_t)(w.part_base + i) * p.hq + head) * D + d;
      *reinterpret_cast<float2*>(dst) = make_float2(v0, v1);
    }
  };
  auto emit_lse = [&](int r, float m, float l) {
    if (r >= rows) return;
    const int i = r / g, j = r % g;
    const int head = kvh * g + j;
    const float lse = (l > 0.f) ? (m + log2f(l)) * kLn2 : -INFINITY;
    if (w.part_base < 0) {
      if (p.lse) p.lse[(int64_t)p.qlist[w.q_off + i] * p.hq + head] = lse;
    } else {
      p.mid_lse[(int64_t)(w.part_base + i) * p.hq + head] = lse;
    }
  };

  if constexpr (NWK == 1) {
    const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      const int d = i * 8 + 2 * (lane % 4);
      emit(r0, d, o[i][0] * inv0, o[i][1] * inv0);
      emit(r1, d, o[i][2] * inv1, o[i][3] * inv1);
    }
    if (lane % 4 == 0) {
      emit_lse(r0, m0, l0);
      emit_lse(r1, m1, l1);
    }
  } else {
    // Combine the NWK warps' partial states (same 16 rows) through shared memory.
    float* sO = reinterpret_cast<float*>(sKV);              // [NWK][16][D]
    float* sM = sO + NWK * 16 * D;                          // [NWK][16]
    float* sL = sM + NWK * 16;
    const int lr0 = lane / 4, lr1 = lr0 + 8;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      const int d = i * 8 + 2 * (lane % 4);
      *reinterpret_cast<float2*>(&sO[(warp_k * 16 + lr0) * D + d]) = make_float2(o[i][0], o[i][1]);
      *reinterpret_cast<float2*>(&sO[(warp_k * 16 + lr1) * D + d]) = make_float2(o[i][2], o[i][3]);
    }
    if (lane % 4 == 0) {
      sM[warp_k * 16 + lr0] = m0; sL[warp_k * 16 + lr0] = l0;
      sM[warp_k * 16 + lr1] = m1; sL[warp_k * 16 + lr1] = l1;
    }
    __syncthreads();
    for (int idx = tid; idx < 16 * (D / 2); idx += 128) {
      const int r = idx / (D / 2), d = (idx % (D / 2)) * 2;
      float mt = -INFINITY;
#pragma unroll
      for (int k = 0; k < NWK; ++k) mt = fmaxf(mt, sM[k * 16 + r]);
      float lt = 0.f, v0 = 0.f, v1 = 0.f;
#pragma unroll
      for (int k = 0; k < NWK; ++k) {
        const float wk = (mt == -INFINITY) ? 0.f : exp2f(sM[k * 16 + r] - mt);
        lt += wk * sL[k * 16 + r];
        v0 += wk * sO[(k * 16 + r) * D + d];
        v1 += wk * sO[(k * 16 + r) * D + d + 1];
      }
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      emit(r, d, v0 * inv, v1 * inv);
      if (d == 0) emit_lse(r, mt, lt);
    }
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(128) attn_tc_kernel(AttnParams p) {
  extern __shared__ __align__(128) char smem[];
  resolve_plan(p);
  if ((int)blockIdx.x >= plan_n_work(p)) return;
  const Work w = p.work[blockIdx.x];
  const int kvh = blockIdx.y;
  if ((int)blockIdx.x < plan_n_wide(p))
    attn_tile<T, D, 64>(p, w, kvh, smem);
  else
    attn_tile<T, D, 16>(p, w, kvh, smem);
}

// CUDA-core path (fp32 pool): a warp per row, lanes across head_dim.
template <typename T>
__global__ void __launch_bounds__(128) attn_simt_kernel(AttnParams p, int D) {
  resolve_plan(p);
  if ((int)blockIdx.x >= plan_n_work(p)) return;
  const Work w = p.work[blockIdx.x];
  const int kvh = blockIdx.y;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int g = p.g;
  const int rows = w.q_len * g;
  const bool causal = (w.flags & BE_WORK_CAUSAL) != 0;
  const int64_t vofs = (int64_t)p.page_size * p.hkv * D;
  const float scale = p.scale_log2 / kLog2e;
  for (int r = warp; r < rows; r += 4) {
    const int i = r / g, j = r % g;
    const int head = kvh * g + j;
    const int qi = p.qlist[w.q_off + i];
    const T* qrow = reinterpret_cast<const T*>(p.q) + qi * p.q_row_stride + (int64_t)head * D;
    float qv[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) qv[k] = (lane + 32 * k < D) ? to_f(qrow[lane + 32 * k]) : 0.f;
    int lim = w.kv_end;
    if (causal) lim = min(lim, w.kv_total - w.q_len + i + 1);
    float m = -INFINITY, l = 0.f, acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int t = w.kv_begin; t < lim; ++t) {
      bool ok;
      const int64_t row = token_row(p, w, t, kvh, D, ok);
      if (!ok) {
        if (lane == 0) flag_range_error();
        continue;
      }
      const T* krow = reinterpret_cast<const T*>(p.pool) + row;
      float dot = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (lane + 32 * k < D) dot += qv[k] * to_f(krow[lane + 32 * k]);
#pragma unroll
      for (int off = 16; off; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
      const float x = dot * scale;
      const float mn = fmaxf(m, x);
      const float a = expf(m - mn);
      const float e = expf(x - mn);
      l = l * a + e;
      const T* vrow = krow + vofs;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (lane + 32 * k < D) acc[k] = acc[k] * a + e * to_f(vrow[lane + 32 * k]);
      m = mn;
    }
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const float lse = l > 0.f ? m + logf(l) : -INFINITY;
    if (w.part_base < 0) {
      T* dst = reinterpret_cast<T*>(p.out) + qi * p.out_row_stride + (int64_t)head * D;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (lane + 32 * k < D) dst[lane + 32 * k] = from_f<T>(acc[k] * inv);
      if (p.lse && lane == 0) p.lse[(int64_t)qi * p.hq + head] = lse;
    } else {
      float* dst = p.mid_o + ((int64_t)(w.part_base + i) * p.hq + head) * D;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (lane + 32 * k < D) dst[lane + 32 * k] = acc[k] * inv;
      if (lane == 0) p.mid_lse[(int64_t)(w.part_base + i) * p.hq + head] = lse;
    }
  }
}

// LSE merge: one warp per (query, head).  Lanes hold head_dim in float4
// chunks; partial rows are read four at a time with independent loads, and
// the log-sum-exp weights come from a lane-parallel pass over the lse values.
template <typename T>
__global__ void __launch_bounds__(128) merge_kernel(const int32_t* __restrict__ mq,
                                                    const int32_t* __restrict__ mptr,
                                                    const int32_t* __restrict__ mparts, int n_merge,
                                                    const float* __restrict__ mid_o,
                                                    const float* __restrict__ mid_lse, int hq, int D,
                                                    char* out, int64_t out_row_stride, float* lse,
                                                    const int32_t* __restrict__ hdr) {
  pdl_wait();
  const int item = blockIdx.x * 4 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (hdr) {
    n_merge = hdr[4];
    mq = hdr + hdr[8];
    mptr = hdr + hdr[9];
    mparts = hdr + hdr[10];
  }
  if (item >= n_merge * hq) return;
  const int b = item / hq, head = item % hq;
  const int qi = mq[b];
  const int p0 = mptr[b], p1 = mptr[b + 1];
  // lane k holds part k's row index and lse (parts beyond 32 are re-read)
  const int np = p1 - p0;
  const int my_row = lane < np ? mparts[p0 + lane] : 0;
  const float my_lse = lane < np ? mid_lse[(int64_t)my_row * hq + head] : -INFINITY;
  float mx = my_lse;
  for (int k = p0 + 32 + lane; k < p1; k += 32) mx = fmaxf(mx, mid_lse[(int64_t)mparts[k] * hq + head]);
#pragma unroll
  for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  T* dst = reinterpret_cast<T*>(out) + qi * out_row_stride + (int64_t)head * D;
  if (mx == -INFINITY) {
    for (int d = lane; d < D; d += 32) dst[d] = from_f<T>(0.f);
    if (lse && lane == 0) lse[(int64_t)qi * hq + head] = -INFINITY;
    return;
  }
  const float my_w = lane < np ? expf(my_lse - mx) : 0.f;
  float den = my_w;
  for (int k = p0 + 32 + lane; k < p1; k += 32) den += expf(mid_lse[(int64_t)mparts[k] * hq + head] - mx);
#pragma unroll
  for (int off = 16; off; off >>= 1) den += __shfl_xor_sync(0xffffffffu, den, off);
  const int nv = D / 4;                 // float4 chunks per row (<= 64)
  float4 acc[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
  for (int k0 = 0; k0 < np; k0 += 8) {
    float wgt[8];
    int64_t row[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int k = k0 + u;
      if (k < 32) {
        wgt[u] = __shfl_sync(0xffffffffu, my_w, k & 31);
        row[u] = __shfl_sync(0xffffffffu, my_row, k & 31);
      } else if (k < np) {
        row[u] = mparts[p0 + k];
        wgt[u] = expf(mid_lse[row[u] * hq + head] - mx);
      } else {
        wgt[u] = 0.f;
        row[u] = 0;
      }
      if (k >= np) wgt[u] = 0.f;
    }
    float4 v[8][2];
#pragma unroll
    for (int u = 0; u < 8; ++u)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int c = lane + 32 * h;
        // parts of weight 0 (LSE -inf: empty, or folded into another part) are not read
        v[u][h] = (k0 + u < np && c < nv && wgt[u] != 0.f)
                      ? __ldg(reinterpret_cast<const float4*>(mid_o + (row[u] * hq + head) * D) + c)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
    for (int u = 0; u < 8; ++u)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        acc[h].x += wgt[u] * v[u][h].x; acc[h].y += wgt[u] * v[u][h].y;
        acc[h].z += wgt[u] * v[u][h].z; acc[h].w += wgt[u] * v[u][h].w;
      }
  }
  const float inv = 1.f / den;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int c = lane + 32 * h;
    if (c < nv) {
      T* o4 = dst + c * 4;
      o4[0] = from_f<T>(acc[h].x * inv); o4[1] = from_f<T>(acc[h].y * inv);
      o4[2] = from_f<T>(acc[h].z * inv); o4[3] = from_f<T>(acc[h].w * inv);
    }
  }
  if (lse && lane == 0) lse[(int64_t)qi * hq + head] = mx + logf(den);
}

template <typename T, int D>
int launch_tc(const AttnParams& p, int n_items, cudaStream_t st) {
  const size_t smem = 64 * D * 2 + 2 * 2 * KT * D * 2;
  static bool attr_set = false;  // per process; the attribute is per function
  if (!attr_set) {
    BE_CUDA_CHECK(cudaFuncSetAttribute(attn_tc_kernel<T, D>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_set = true;
  }
  dim3 grid(n_items, p.hkv);
  attn_tc_kernel<T, D><<<grid, 128, smem, st>>>(p);
  BE_LAUNCH_CHECK();
  return BE_OK;
}

}  // namespace be

