// Beam-tile decode attention on the 5th-generation tensor cores.
//
// A tile is up to M = 64 or 128 query-head rows (one prompt's beams x the g
// query heads of one KV head).  Everything the tile's beams attend -- the
// shared prompt, the shared branches and every beam's own suffix -- is one
// list of page entries (page, valid tokens, query range).  A CTA takes one
// piece (a range of the list) and one KV head and streams it in chunks of
// four pages:
//
//   warp 4 (producer)  page entries -> shared memory, TMA loads of the K and V
//                      boxes (16 tokens x 64 dims, 128-byte swizzle) into a
//                      ring of TL_NS stages;
//   warp 5 (MMA)       S = Q K^T (M x 64 tokens, tcgen05.mma kind::f16, fp32 in
//                      TMEM, double-buffered), then O += P V (M x 128 dims in
//                      TMEM) once the softmax has written P;
//   warps 0-3          one thread per row: S from TMEM, the entry masks (row's
//                      query inside the page's query range, slot < valid
//                      tokens), online softmax with a lazy rescale (O in TMEM
//                      is rescaled only when a row's max grows by more than
//                      2^8), P in bf16/f16 into the stage's K area; at the end
//                      O / l to the output, or a partial row (O / l and the
//                      LSE) when the tile has several pieces.
//
// tile_merge_kernel (launched right after, programmatic dependent launch)
// merges the partial rows of multi-piece tiles by LSE, one warp per row over
// all SMs.
//
// Each page is read once per KV head; a suffix page's scores are computed for
// every row of the tile and masked for the rows of other beams (tensor-core
// work is cheap here, HBM bytes are not).  All waits are bounded: on expiry
// the CTA records BE_EDEVICE_TIMEOUT, stops issuing work, drains what it
// issued and frees its TMEM.
namespace be {

constexpr int TL_PAGES = 4;                    // pages per chunk
constexpr int TL_CHUNK = TL_PAGES * 16;        // tokens per chunk (page size 16)
constexpr int TL_KHALF = TL_CHUNK * 128;       // one 64-dim half of K or V: 64 rows x 128 B
constexpr int TL_KV = 2 * TL_KHALF;            // K (or V) of a chunk, 16 KB
constexpr int TL_STAGE = 2 * TL_KV;            // K + V
constexpr int TL_TMEM_COLS = 256;              // S (2 x 64 columns) | O (128 columns)
constexpr uint32_t TL_O_COL = 128;

template <int M>
struct TileShape {
  static constexpr int NS = M == 64 ? 3 : 2;   // pipeline stages (two CTAs per SM either way)
  static constexpr int QHALF = M * 128;        // one 64-dim half of Q: M rows x 128 B
  static constexpr size_t smem() {
    // no alignment slack: two CTAs per SM need every byte; the kernel checks
    // that the dynamic shared memory starts on a 1024-byte boundary
    return 2 * QHALF + (size_t)NS * TL_STAGE + NS * TL_PAGES * 16 + 256;
  }
};

struct TileParams {
  const int32_t* plan;
  const char* q;
  int64_t q_row_stride;  // elements
  int num_pages, hq, hkv, g;
  float scale_log2;
  char* out;
  int64_t out_row_stride;
  float* lse;
  void* part_o;          // [part pieces][hkv][M][128] of T
  float* part_lse;
  int max_part_pieces, max_tiles;
  int plan_early;
  int cluster;           // > 1: CTAs of a (tile, KV head) form a cluster, merged on chip
  int merge_next;        // tile_merge_kernel follows on the stream
  int debug;             // BE_ATTN_DEBUG & 4: globaltimer stamps into lse (per CTA x 16)
};

template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t v);
template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t v) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v));
}
template <>
__device__ __forceinline__ float2 unpack2<__half>(uint32_t v) {
  return __half22float2(*reinterpret_cast<const __half2*>(&v));
}

// Non-blocking phase test (try_wait may suspend the thread for a while when the
// phase is not complete; the MMA issuer polls two barriers and must not).
__device__ __forceinline__ bool mbar_test(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Warp-uniform bounded wait: lane 0 waits, the warp follows its verdict.
__device__ __forceinline__ bool tl_warp_wait(uint64_t* b, uint32_t parity) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(b, parity);
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// tcgen05.ld / st of 16 TMEM lanes x 64 columns (".16x256b.x8"): thread t gets
// lanes t/4 and t/4 + 8, columns 8j + 2(t%4) + {0, 1} of blocks j = 0..7, as
// r[4j], r[4j+1] (lane t/4) and r[4j+2], r[4j+3] (lane t/4 + 8) -- the layout
// of an M = 64 accumulator's 16 rows per warp, with every thread holding data.
__device__ __forceinline__ void tmem_ld16x8(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16x8(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x256b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// Four 8x8 b16 matrices to shared memory; register i of thread t holds row t/4,
// columns 2(t%4), 2(t%4)+1 of matrix i; threads 8i..8i+7 give matrix i's row
// addresses.
__device__ __forceinline__ void stmatrix4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                          uint32_t d) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr),
               "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}
__device__ __forceinline__ float4 ld_peer4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ float quad_max(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
  return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
}
__device__ __forceinline__ float quad_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  return v + __shfl_xor_sync(0xffffffffu, v, 2);
}

__device__ __forceinline__ void tstamp(const TileParams& p, int k) {
  if ((p.debug & 4) && p.lse)
    reinterpret_cast<unsigned long long*>(p.lse)[((int64_t)blockIdx.y * gridDim.x + blockIdx.x) * 64 +
                                                 k] = gtimer();
}

// LSE merge of one row (128 dims) over a tile's pieces by one warp: lane =
// piece group (G of them) x segment (32 / G segments of 4 G dims).  A step
// takes four pieces of the lane's group, k, k + G, k + 2G, k + 3G: their LSEs
// and partial rows are loaded together (one round trip for up to 4 G pieces),
// then folded with a running max; rows a piece did not see (LSE -inf, never
// written) are selected away.  The groups combine through shuffles.
template <typename T, int G>
__device__ __forceinline__ void merge_row_warp(const TileParams& p, int part_base, int npieces,
                                               int kvh, int M, int rr, int q_row, int head) {
  constexpr int SEG = 32 / G, DIMS = 4 * G, V = DIMS / 8;   // int4 vectors per piece
  const int lane = threadIdx.x & 31, grp = lane / SEG, seg = lane % SEG;
  float m = -INFINITY, wsum = 0.f;
  float acc[DIMS];
#pragma unroll
  for (int i = 0; i < DIMS; ++i) acc[i] = 0.f;
  const T* po = reinterpret_cast<const T*>(p.part_o);
  for (int k = grp; k < npieces; k += 4 * G) {
    float l[4];
    int4 x[4][V];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int kk = min(k + G * u, npieces - 1);
      const int64_t row = ((int64_t)(part_base + kk) * p.hkv + kvh) * M + rr;
      l[u] = (k + G * u < npieces) ? __ldcg(p.part_lse + row) : -INFINITY;
      const int4* src = reinterpret_cast<const int4*>(po + row * 128 + seg * DIMS);
#pragma unroll
      for (int i = 0; i < V; ++i) x[u][i] = __ldcg(src + i);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (!(l[u] > -INFINITY)) continue;
      const float mn = fmaxf(m, l[u]);
      const float a = ex2(m - mn), w = ex2(l[u] - mn);   // m = -inf: a = 0
      m = mn;
      wsum = wsum * a + w;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const uint32_t* h = reinterpret_cast<const uint32_t*>(&x[u][i]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = unpack2<T>(h[q]);
          acc[8 * i + 2 * q] = acc[8 * i + 2 * q] * a + w * f.x;
          acc[8 * i + 2 * q + 1] = acc[8 * i + 2 * q + 1] * a + w * f.y;
        }
      }
    }
  }
  float mall = m;
#pragma unroll
  for (int o = SEG; o < 32; o <<= 1) mall = fmaxf(mall, __shfl_xor_sync(0xffffffffu, mall, o));
  const float sc = mall > -INFINITY && m > -INFINITY ? ex2(m - mall) : 0.f;
  wsum *= sc;
#pragma unroll
  for (int i = 0; i < DIMS; ++i) acc[i] *= sc;
#pragma unroll
  for (int o = SEG; o < 32; o <<= 1) {
    wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
#pragma unroll
    for (int i = 0; i < DIMS; ++i) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
  }
  if (grp != 0) return;
  const float iw = wsum > 0.f ? 1.f / wsum : 0.f;
  T* dst = reinterpret_cast<T*>(p.out) + (int64_t)q_row * p.out_row_stride + (int64_t)head * 128 +
           seg * DIMS;
#pragma unroll
  for (int k = 0; k < DIMS; k += 8) {
    uint32_t w4[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) w4[u] = pack2<T>(acc[k + 2 * u] * iw, acc[k + 2 * u + 1] * iw);
    *reinterpret_cast<int4*>(dst + k) = make_int4(w4[0], w4[1], w4[2], w4[3]);
  }
  if (seg == 0 && p.lse && !(p.debug & 4))
    p.lse[(int64_t)q_row * p.hq + head] = wsum > 0.f ? (mall + log2f(wsum)) * kLn2 : -INFINITY;
}

template <typename T, int M>
__global__ void __launch_bounds__(192, 2) attn_tile_kernel(const __grid_constant__ CUtensorMap tmap,
                                                        TileParams p) {
  using S_ = TileShape<M>;
  constexpr int NS = S_::NS, QHALF = S_::QHALF;
  extern __shared__ __align__(1024) char smem_raw[];
  if (smem_u32(smem_raw) & 1023) {                  // swizzled operands need 1024-B atoms
    if (threadIdx.x == 0) flag_range_error();
    return;
  }
  char* sQ = smem_raw;                              // [2 halves][M rows][128 B]
  char* sStage = sQ + 2 * QHALF;                    // [NS][K 16 KB (then P) | V 16 KB]
  int4* sMeta = reinterpret_cast<int4*>(sStage + NS * TL_STAGE);   // [NS][4] entries
  uint64_t* bars = reinterpret_cast<uint64_t*>(sMeta + NS * TL_PAGES);
  uint64_t* kfull = bars;                 // [NS] K boxes (+ entries) landed
  uint64_t* vfull = bars + NS;            // [NS] V boxes landed
  uint64_t* sfree = bars + 2 * NS;        // [NS] stage consumed by its PV MMAs
  uint64_t* sfull = bars + 3 * NS;        // [2]  S tile in TMEM
  uint64_t* pready = bars + 3 * NS + 2;   // [2]  P written (128 softmax threads)
  uint64_t* odone = bars + 3 * NS + 4;    // O += P V of a chunk completed
  uint64_t* qfull = bars + 3 * NS + 5;    // Q in shared memory (128 threads)
  uint64_t* drain = bars + 3 * NS + 6;    // abort path: every issued MMA completed
  // the last O += P V completed.  (A parity wait on `odone` cannot tell the last
  // completion from the one before it: two PV products may be in flight when
  // the softmax finishes its last chunk.)
  uint64_t* ofinal = bars + 3 * NS + 7;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(bars + 3 * NS + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* issued = abort_flag + 1;  // chunks whose loads the producer issued

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kvh = blockIdx.y;
  if (tid == 0) tstamp(p, 0);
  if (!p.plan_early) pdl_wait();
  const int32_t* hdr = p.plan;
  const int pi = blockIdx.x;
  // one round trip: the header and this CTA's piece (pieces sit right after the header)
  const int4 h0 = __ldg(reinterpret_cast<const int4*>(hdr));       // n_tiles, n_pieces, ...
  const int4 h1 = __ldg(reinterpret_cast<const int4*>(hdr) + 1);   // ..., off_entries, total
  const int4* pcs = reinterpret_cast<const int4*>(hdr + BE_PLAN_HEADER_INTS) + 6 * pi;
  const int4 pc = __ldg(pcs), pq = __ldg(pcs + 1);
  if (pi >= h0.y) return;                           // before any barrier or TMEM use
  const int plan_cluster = __ldg(hdr + 14);
  if (plan_cluster != (p.cluster > 1 ? p.cluster : 0)) {   // uniform over the grid
    if (tid == 0 && pi == 0 && kvh == 0) flag_range_error();
    return;
  }
  const bool on_chip = p.cluster > 1;              // pieces merged through DSMEM
  const int tile = pc.x, ent_begin = pc.y, ent_end = pc.z, kidx = pc.w;
  const int q_begin = pq.x, q_len = pq.y, t_npieces = pq.z, part_base = pq.w;
  const int4* ents = reinterpret_cast<const int4*>(hdr + h1.z);
  const int g = p.g, rows = min(q_len * g, M);
  const int n_ent = max(0, ent_end - ent_begin);
  const int nch = (n_ent + TL_PAGES - 1) / TL_PAGES;
  if (!on_chip && t_npieces > 1 && (part_base < 0 || part_base + kidx >= p.max_part_pieces ||
                                    tile >= p.max_tiles)) {   // slot outside the caller's buffers
    if (tid == 0) flag_range_error();
    return;
  }

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(kfull + s, 1);
      mbar_init(vfull + s, 1);
      mbar_init(sfree + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(sfull + b, 1);
      mbar_init(pready + b, 128);
    }
    mbar_init(odone, 1);
    mbar_init(qfull, 128);
    mbar_init(drain, 1);
    mbar_init(ofinal, 1);
    *abort_flag = 0;
    *issued = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 5) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32((const void*)tmem_slot)), "n"(TL_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) tstamp(p, 1);
  if (p.plan_early) pdl_wait();                      // q and the pages come from earlier kernels
  if (tid == 0) tstamp(p, 2);

  if (warp == 4) {
    // ---------------- producer ----------------
    // the piece's first 128 entries in registers (lane l holds entries l, l+32, ...)
    if (lane == 0) asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap) : "memory");
    int4 pre[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {   // chunk 0's entries come with the piece record
      const int j = u * 32 + lane;
      pre[u] = j < n_ent ? __ldg(j < TL_PAGES ? pcs + 2 + j : ents + ent_begin + j)
                         : make_int4(0, 0, 0, 0);
    }
    for (int c = 0; c < nch; ++c) {
      const int s = c % NS;
      if (c >= NS && !tl_warp_wait(sfree + s, ((c / NS) - 1) & 1)) {
        *abort_flag = 1;
        break;
      }
      if (*abort_flag) break;
      const int j0 = c * TL_PAGES;
      const int npg = min(TL_PAGES, n_ent - j0);
      // lanes holding this chunk's entries write them to the stage's metadata
      int4 e = make_int4(0, 0, 0, 0);
      bool mine = false;
      int slot = 0;
      if (j0 + TL_PAGES <= 128) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int j = u * 32 + lane;
          if (j >= j0 && j < j0 + npg) {
            e = pre[u];
            mine = true;
            slot = j - j0;
          }
        }
      } else if (lane < npg) {
        e = __ldg(ents + ent_begin + j0 + lane);
        mine = true;
        slot = lane;
      }
      if (mine) {
        if (e.x < 0 || e.x >= p.num_pages || e.y < 0 || e.y > 16) {
          flag_range_error();
          e = make_int4(0, 0, 0, 0);   // page 0, no valid tokens: read but masked
        }
        sMeta[s * TL_PAGES + slot] = e;
      }
      if (lane >= npg && lane < TL_PAGES) sMeta[s * TL_PAGES + lane] = make_int4(0, 0, 0, 0);
      __syncwarp();
      if (lane == 0) {
        char* sK = sStage + s * TL_STAGE;
        char* sV = sK + TL_KV;
        mbar_expect_tx(kfull + s, npg * 2 * TMA_BOX_BYTES);   // arrive: releases sMeta too
        for (int j = 0; j < npg; ++j) {
          const int page = sMeta[s * TL_PAGES + j].x;
#pragma unroll
          for (int h = 0; h < 2; ++h)
            tma_load5(smem_u32(sK + h * TL_KHALF + j * TMA_BOX_BYTES), &tmap, kfull + s, h * 64,
                      kvh, 0, 0, page);
        }
        mbar_expect_tx(vfull + s, npg * 2 * TMA_BOX_BYTES);
        for (int j = 0; j < npg; ++j) {
          const int page = sMeta[s * TL_PAGES + j].x;
#pragma unroll
          for (int h = 0; h < 2; ++h)
            tma_load5(smem_u32(sV + h * TL_KHALF + j * TMA_BOX_BYTES), &tmap, vfull + s, h * 64,
                      kvh, 0, 1, page);
        }
        *issued = c + 1;
        if (c < 8) tstamp(p, 40 + c);
      }
      __syncwarp();
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    // Event-driven: S(cs) as soon as K(cs) landed and its TMEM buffer is free
    // (at most two S tiles ahead of the PV products), O += P V of chunk cp as
    // soon as the softmax wrote P(cp) and V(cp) landed.
    if (lane == 0 && nch > 0) {
      bool ok = mbar_wait(qfull, 0);
      int cs = 0, cp = 0;
      uint64_t t0 = 0;
      uint32_t idle = 0;
      while (ok && cp < nch) {
        bool progressed = false;
        if (cs < nch && cs < cp + 2 && mbar_test(kfull + cs % NS, (cs / NS) & 1)) {
          const int s = cs % NS, b = cs & 1;
          tc_fence_after();
          const int npg = min(TL_PAGES, n_ent - cs * TL_PAGES);
          const uint32_t idesc = umma_idesc<T>(M, 16 * npg, 0);
          char* sK = sStage + s * TL_STAGE;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const int h = kk >> 2, koff = (kk & 3) * 32;
            const uint64_t a = umma_desc(smem_u32(sQ + h * QHALF) + koff, 16, 1024);
            const uint64_t bd = umma_desc(smem_u32(sK + h * TL_KHALF) + koff, 16, 1024);
            umma_f16(tmem + b * TL_CHUNK, a, bd, idesc, kk > 0 ? 1u : 0u);
          }
          umma_commit(sfull + b);
          if (cs < 8) tstamp(p, 24 + cs);
          ++cs;
          progressed = true;
        }
        if (cp < cs && mbar_test(pready + (cp & 1), (cp >> 1) & 1) &&
            mbar_test(vfull + cp % NS, (cp / NS) & 1)) {
          const int s = cp % NS;
          tc_fence_after();
          const int npg = min(TL_PAGES, n_ent - cp * TL_PAGES);
          const uint32_t idesc = umma_idesc<T>(M, 128, 1);
          char* sP = sStage + s * TL_STAGE;
          char* sV = sP + TL_KV;
          for (int j = 0; j < npg; ++j) {
            const uint64_t a = umma_desc(smem_u32(sP) + j * 32, 16, 1024);
            const uint64_t bd = umma_desc(smem_u32(sV + j * TMA_BOX_BYTES), TL_KHALF, 1024);
            umma_f16(tmem + TL_O_COL, a, bd, idesc, (cp > 0 || j > 0) ? 1u : 0u);
          }
          umma_commit(odone);
          umma_commit(sfree + s);
          if (cp == nch - 1) umma_commit(ofinal);
          if (cp < 8) tstamp(p, 32 + cp);
          ++cp;
          progressed = true;
        }
        if (progressed) {
          t0 = 0;
          idle = 0;
        } else if ((++idle & 255) == 0) {   // bounded: no progress for kWaitNs
          const uint64_t t = gtimer();
          if (t0 == 0) {
            t0 = t;
          } else if (t - t0 > kWaitNs || *abort_flag) {
            atomicCAS(&g_device_status, 0, BE_EDEVICE_TIMEOUT);
            ok = false;
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        umma_commit(drain);              // arrives once every MMA issued so far completed
        mbar_wait(drain, 0);
        // release the softmax warps from their waits so the CTA can drain
        for (int b = 0; b < 2; ++b) mbar_arrive(sfull + b);
        mbar_arrive(odone);
        mbar_arrive(ofinal);
      }
    }
    __syncwarp();
  } else {
    // ---------------- softmax / epilogue (warps 0-3) ----------------
    // Q rows -> shared memory, K-major with the 128-byte swizzle
    {
      constexpr int QN = M * 16 / 128;               // 16-byte vectors per thread
      int4 qv[QN];
#pragma unroll
      for (int u = 0; u < QN; ++u) {                 // all loads in flight, then the stores
        const int idx = tid + u * 128, r = idx >> 4, c = idx & 15;
        qv[u] = make_int4(0, 0, 0, 0);
        if (r < rows)
          qv[u] = __ldg(reinterpret_cast<const int4*>(
              reinterpret_cast<const T*>(p.q) + (int64_t)(q_begin + r / g) * p.q_row_stride +
              (int64_t)(kvh * g + r % g) * 128 + c * 8));
      }
#pragma unroll
      for (int u = 0; u < QN; ++u) {
        const int idx = tid + u * 128, r = idx >> 4, c = idx & 15;
        *reinterpret_cast<int4*>(sQ + (c >> 3) * QHALF + r * 128 + (((c & 7) ^ (r & 7)) << 4)) =
            qv[u];
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_arrive(qfull);

    if constexpr (M == 64) {
      // 16 rows per warp in the 16x256b layout: rows rA = 16 w + lane / 4 and
      // rB = rA + 8, columns 2 (lane % 4) + {0, 1} of each 8-column block; the
      // four threads of a row combine maxima with shuffles, and keep partial sums
      const int rA = warp * 16 + (lane >> 2), rB = rA + 8, cp = lane & 3;
      const bool okA = rA < rows, okB = rB < rows;
      const int qA = okA ? rA / g : -1, qB = okB ? rB / g : -1;
      const uint32_t tw = tmem + ((uint32_t)(warp * 32) << 16);
      float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
      bool alive = true;
      for (int c = 0; c < nch; ++c) {
        const int s = c % NS, b = c & 1;
        if (!tl_warp_wait(kfull + s, (c / NS) & 1) || !tl_warp_wait(sfull + b, (c >> 1) & 1) ||
            *abort_flag) {
          alive = false;
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        if (tid == 0 && c < 8) tstamp(p, 8 + c);
        if (tid == 0 && c == 0) tstamp(p, 3);
        int limA[TL_PAGES], limB[TL_PAGES];
        bool partial = false;
        const int npg = min(TL_PAGES, ent_end - (ent_begin + c * TL_PAGES));
#pragma unroll
        for (int j = 0; j < TL_PAGES; ++j) {
          const int4 e = sMeta[s * TL_PAGES + j];
          limA[j] = (j < npg && qA >= e.z && qA < e.w) ? e.y : 0;
          limB[j] = (j < npg && qB >= e.z && qB < e.w) ? e.y : 0;
          partial |= j < npg && e.y < 16;
        }
        uint32_t v[32];
        tmem_ld16x8(tw + b * TL_CHUNK, v);
        tmem_wait();
        if (tid == 0 && c < 4) tstamp(p, 48 + c);
        float xa[16], xb[16];
#pragma unroll
        for (int jb = 0; jb < 8; ++jb)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int slot = ((jb & 1) << 3) + 2 * cp + e, pg = jb >> 1;
            xa[2 * jb + e] = slot < limA[pg] ? __uint_as_float(v[4 * jb + e]) * p.scale_log2
                                             : -INFINITY;
            xb[2 * jb + e] = slot < limB[pg] ? __uint_as_float(v[4 * jb + 2 + e]) * p.scale_log2
                                             : -INFINITY;
          }
        float ta[8], tb[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          ta[i] = fmaxf(xa[i], xa[i + 8]);
          tb[i] = fmaxf(xb[i], xb[i + 8]);
        }
#pragma unroll
        for (int w = 4; w >= 1; w >>= 1)
#pragma unroll
          for (int i = 0; i < w; ++i) {
            ta[i] = fmaxf(ta[i], ta[i + w]);
            tb[i] = fmaxf(tb[i], tb[i + w]);
          }
        const float mxA = quad_max(ta[0]), mxB = quad_max(tb[0]);
        const bool growA = mxA > mA + 8.f, growB = mxB > mB + 8.f;
        const bool rescA = growA && mA > -INFINITY, rescB = growB && mB > -INFINITY;
        const float alA = rescA ? ex2(mA - mxA) : 1.f, alB = rescB ? ex2(mB - mxB) : 1.f;
        if (growA) mA = mxA;
        if (growB) mB = mxB;
        const float muA = mA > -INFINITY ? mA : 0.f, muB = mB > -INFINITY ? mB : 0.f;
        uint32_t pa[8], pb[8];
        float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int jb = 0; jb < 8; ++jb) {
          const float a0 = ex2(xa[2 * jb] - muA), a1 = ex2(xa[2 * jb + 1] - muA);
          const float b0 = ex2(xb[2 * jb] - muB), b1 = ex2(xb[2 * jb + 1] - muB);
          sa[jb & 3] += a0 + a1;
          sb[jb & 3] += b0 + b1;
          pa[jb] = pack2<T>(a0, a1);
          pb[jb] = pack2<T>(b0, b1);
        }
        lA = lA * alA + ((sa[0] + sa[1]) + (sa[2] + sa[3]));
        lB = lB * alB + ((sb[0] + sb[1]) + (sb[2] + sb[3]));
        if (tid == 0 && c < 4) tstamp(p, 52 + c);
        if (c > 0 && __any_sync(0xffffffffu, rescA || rescB)) {
          if (!tl_warp_wait(odone, (c - 1) & 1)) {
            alive = false;
            *abort_flag = 1;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t o[32];
            tmem_ld16x8(tw + TL_O_COL + 64 * h, o);
            tmem_wait();
#pragma unroll
            for (int jb = 0; jb < 8; ++jb) {
              o[4 * jb] = __float_as_uint(__uint_as_float(o[4 * jb]) * alA);
              o[4 * jb + 1] = __float_as_uint(__uint_as_float(o[4 * jb + 1]) * alA);
              o[4 * jb + 2] = __float_as_uint(__uint_as_float(o[4 * jb + 2]) * alB);
              o[4 * jb + 3] = __float_as_uint(__uint_as_float(o[4 * jb + 3]) * alB);
            }
            tmem_st16x8(tw + TL_O_COL + 64 * h, o);
          }
          tmem_wait_st();
        }
        {   // P (bf16 / f16) into the stage's K area, K-major with the 128-byte swizzle
          char* sP = sStage + s * TL_STAGE;
          const int mi = lane >> 3, rr = lane & 7;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int jb = 2 * k + (mi >> 1), row = warp * 16 + ((mi & 1) << 3) + rr;
            stmatrix4(smem_u32(sP + row * 128 + ((jb ^ (row & 7)) << 4)), pa[2 * k], pb[2 * k],
                      pa[2 * k + 1], pb[2 * k + 1]);
          }
        }
        if (tid == 0 && c < 4) tstamp(p, 56 + c);
        if (partial) {
          if (!tl_warp_wait(vfull + s, (c / NS) & 1)) {
            alive = false;
            *abort_flag = 1;
            break;
          }
          char* sV = sStage + s * TL_STAGE + TL_KV;
          for (int idx = tid; idx < TL_PAGES * 16 * 16; idx += 128) {
            const int j = idx >> 8, t = (idx >> 4) & 15, ch = idx & 15;
            if (j < npg && t >= sMeta[s * TL_PAGES + j].y)
              *reinterpret_cast<int4*>(sV + (ch >> 3) * TL_KHALF + (j * 16 + t) * 128 +
                                       (ch & 7) * 16) = make_int4(0, 0, 0, 0);
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tc_fence_before();
        mbar_arrive(pready + b);
        if (tid == 0 && c < 8) tstamp(p, 16 + c);
      }
      if (tid == 0) tstamp(p, 4);
      if (p.merge_next) pdl_trigger();              // only our merge kernel may start early
      // ---------------- epilogue (M = 64) ----------------
      const bool have_o = alive && nch > 0 && tl_warp_wait(ofinal, 0) && !*abort_flag;
      if (nch > 0 && !have_o) alive = false;
      tc_fence_after();
      lA = quad_sum(lA);
      lB = quad_sum(lB);
      const float invA = lA > 0.f ? 1.f / lA : 0.f, invB = lB > 0.f ? 1.f / lB : 0.f;
      const bool direct = t_npieces <= 1;
      T* dA = nullptr;
      T* dB = nullptr;
      if (direct) {
        dA = reinterpret_cast<T*>(p.out) + (int64_t)(q_begin + (okA ? qA : 0)) * p.out_row_stride +
             (int64_t)(kvh * g + rA % g) * 128;
        dB = reinterpret_cast<T*>(p.out) + (int64_t)(q_begin + (okB ? qB : 0)) * p.out_row_stride +
             (int64_t)(kvh * g + rB % g) * 128;
      } else if (!on_chip) {
        T* base = reinterpret_cast<T*>(p.part_o) +
                  ((int64_t)(part_base + kidx) * p.hkv + kvh) * M * 128;
        dA = base + (int64_t)rA * 128;
        dB = base + (int64_t)rB * 128;
      }
      const bool wA = okA && alive && (direct || lA > 0.f);   // empty partial rows: LSE only
      const bool wB = okB && alive && (direct || lB > 0.f);
      float* sO = reinterpret_cast<float*>(sStage);     // on-chip partial rows [M][128] fp32
      float* sL = reinterpret_cast<float*>(sQ);         // and their log2 LSE [M]
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t o[32];
        if (have_o) {
          tmem_ld16x8(tw + TL_O_COL + 64 * h, o);
          tmem_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
#pragma unroll
        for (int jb = 0; jb < 8; ++jb) {
          const int col = 64 * h + 8 * jb + 2 * cp;
          const float a0 = __uint_as_float(o[4 * jb]) * invA, a1 = __uint_as_float(o[4 * jb + 1]) * invA;
          const float b0 = __uint_as_float(o[4 * jb + 2]) * invB, b1 = __uint_as_float(o[4 * jb + 3]) * invB;
          if (on_chip && !direct) {
            if (wA) *reinterpret_cast<float2*>(sO + rA * 128 + col) = make_float2(a0, a1);
            if (wB) *reinterpret_cast<float2*>(sO + rB * 128 + col) = make_float2(b0, b1);
          } else {
            if (wA) *reinterpret_cast<uint32_t*>(dA + col) = pack2<T>(a0, a1);
            if (wB) *reinterpret_cast<uint32_t*>(dB + col) = pack2<T>(b0, b1);
          }
        }
      }
      if (tid == 0) tstamp(p, 5);
      if (cp == 0 && on_chip && !direct) {   // every row's LSE, -inf when empty or aborted
        sL[rA] = (alive && lA > 0.f) ? mA + log2f(lA) : -INFINITY;
        sL[rB] = (alive && lB > 0.f) ? mB + log2f(lB) : -INFINITY;
      } else if (cp == 0 && alive) {
        const float lse2A = lA > 0.f ? mA + log2f(lA) : -INFINITY;
        const float lse2B = lB > 0.f ? mB + log2f(lB) : -INFINITY;
        if (direct) {
          if (p.lse && !(p.debug & 4)) {
            if (okA) p.lse[(int64_t)(q_begin + qA) * p.hq + kvh * g + rA % g] = lse2A * kLn2;
            if (okB) p.lse[(int64_t)(q_begin + qB) * p.hq + kvh * g + rB % g] = lse2B * kLn2;
          }
        } else {
          float* pl = p.part_lse + ((int64_t)(part_base + kidx) * p.hkv + kvh) * M;
          if (okA) pl[rA] = lse2A;
          if (okB) pl[rB] = lse2B;
        }
      }
    } else {
    // this thread's row and TMEM lane
    const bool lane_ok = M == 128 || lane < 16;
    const int r = M == 128 ? tid : warp * 16 + lane;
    const bool row_ok = lane_ok && r < rows;
    const int qr = row_ok ? r / g : -1;
    const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
    float m_use = -INFINITY, l_sum = 0.f;
    bool alive = true;
    for (int c = 0; c < nch; ++c) {
      const int s = c % NS, b = c & 1;
      if (!tl_warp_wait(kfull + s, (c / NS) & 1) || !tl_warp_wait(sfull + b, (c >> 1) & 1) ||
          *abort_flag) {
        alive = false;
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      if (tid == 0 && c < 8) tstamp(p, 8 + c);
      if (tid == 0 && c == 0) tstamp(p, 3);
      int lim[TL_PAGES];
      bool partial = false;
      const int npg = min(TL_PAGES, ent_end - (ent_begin + c * TL_PAGES));
#pragma unroll
      for (int j = 0; j < TL_PAGES; ++j) {
        const int4 e = sMeta[s * TL_PAGES + j];
        lim[j] = (j < npg && qr >= e.z && qr < e.w) ? e.y : 0;
        partial |= j < npg && e.y < 16;
      }
      uint32_t v[TL_CHUNK];
      tmem_ld32_nw(trow + b * TL_CHUNK, v);
      tmem_ld32_nw(trow + b * TL_CHUNK + 32, v + 32);
      tmem_wait();
      if (tid == 0 && c < 4) tstamp(p, 48 + c);
      // masked scores -> -inf, max by a tree (independent lanes of work per step)
      float x[TL_CHUNK];
#pragma unroll
      for (int i = 0; i < TL_CHUNK; ++i)
        x[i] = ((i & 15) < lim[i >> 4]) ? __uint_as_float(v[i]) * p.scale_log2 : -INFINITY;
      float mt[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) mt[i] = fmaxf(fmaxf(x[i], x[i + 16]), fmaxf(x[i + 32], x[i + 48]));
#pragma unroll
      for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
        for (int i = 0; i < w; ++i) mt[i] = fmaxf(mt[i], mt[i + w]);
      const float mx = mt[0];
      const bool grow = mx > m_use + 8.f;          // also true for the first visible tokens
      // a row without earlier visible tokens has O = 0 and l = 0: nothing to rescale
      const bool rescale = grow && m_use > -INFINITY;
      const float alpha = rescale ? ex2(m_use - mx) : 1.f;
      if (grow) m_use = mx;
      // ex2(-inf - m) = 0 for masked scores (m finite); rows with nothing visible
      // (m = -inf) take 0 everywhere
      const float mu = m_use > -INFINITY ? m_use : 0.f;
      float st[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) st[i] = 0.f;
      uint32_t pk[TL_CHUNK / 2];
#pragma unroll
      for (int i = 0; i < TL_CHUNK; i += 2) {
        const float e0 = ex2(x[i] - mu), e1 = ex2(x[i + 1] - mu);
        st[(i >> 1) & 7] += e0 + e1;
        pk[i / 2] = pack2<T>(e0, e1);
      }
      const float sum = ((st[0] + st[1]) + (st[2] + st[3])) + ((st[4] + st[5]) + (st[6] + st[7]));
      l_sum = l_sum * alpha + sum;
      if (tid == 0 && c < 4) tstamp(p, 52 + c);
      // rows whose max grew: rescale the O accumulated so far (after chunk c-1's PV)
      if (c > 0 && __any_sync(0xffffffffu, rescale)) {
        if (!tl_warp_wait(odone, (c - 1) & 1)) {
          alive = false;
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const float a = alpha;
#pragma unroll
        for (int c0 = 0; c0 < 128; c0 += 32) {
          uint32_t o[32];
          tmem_ld32_nw(trow + TL_O_COL + c0, o);
          tmem_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * a);
          tmem_st32(trow + TL_O_COL + c0, o);
        }
        tmem_wait_st();
      }
      // P row r: 64 tokens = 8 swizzled 16-byte chunks in the stage's K area
      if (lane_ok) {
        char* prow = sStage + s * TL_STAGE + r * 128;
#pragma unroll
        for (int q8 = 0; q8 < 8; ++q8)
          *reinterpret_cast<int4*>(prow + ((q8 ^ (r & 7)) << 4)) =
              make_int4(pk[q8 * 4], pk[q8 * 4 + 1], pk[q8 * 4 + 2], pk[q8 * 4 + 3]);
      }
      if (tid == 0 && c < 4) tstamp(p, 56 + c);
      // V rows past a page's valid tokens: zero (stale pool data may be non-finite)
      if (partial) {
        if (!tl_warp_wait(vfull + s, (c / NS) & 1)) {
          alive = false;
          *abort_flag = 1;
          break;
        }
        char* sV = sStage + s * TL_STAGE + TL_KV;
        for (int idx = tid; idx < TL_PAGES * 16 * 16; idx += 128) {
          const int j = idx >> 8, t = (idx >> 4) & 15, ch = idx & 15;   // page, slot, 16-B chunk
          if (j < npg && t >= sMeta[s * TL_PAGES + j].y)
            *reinterpret_cast<int4*>(sV + (ch >> 3) * TL_KHALF + (j * 16 + t) * 128 +
                                     (ch & 7) * 16) = make_int4(0, 0, 0, 0);
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      mbar_arrive(pready + b);
      if (tid == 0 && c < 8) tstamp(p, 16 + c);
    }
    if (tid == 0) tstamp(p, 4);
    // only our merge kernel may start early: it waits for this grid before reading;
    // another library's kernel launched next may read the output without waiting
    if (p.merge_next) pdl_trigger();
    // ---------------- epilogue ----------------
    const bool have_o = alive && nch > 0 && tl_warp_wait(ofinal, 0) && !*abort_flag;
    if (nch > 0 && !have_o) alive = false;
    tc_fence_after();
    const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
    const float lse2 = l_sum > 0.f ? m_use + log2f(l_sum) : -INFINITY;
    const bool direct = t_npieces <= 1;
    const int head = kvh * g + (row_ok ? r % g : 0);
    const int qi = q_begin + (row_ok ? qr : 0);
    T* prow_o = nullptr;   // partial rows in the pool's 2-byte type
    float* sO = reinterpret_cast<float*>(sStage);     // on-chip partial rows [M][128] fp32
    float* sL = reinterpret_cast<float*>(sQ);         // and their log2 LSE [M]
    if (!direct && !on_chip)
      prow_o = reinterpret_cast<T*>(p.part_o) +
               (((int64_t)(part_base + kidx) * p.hkv + kvh) * M + r) * 128;
#pragma unroll
    for (int c0 = 0; c0 < 128; c0 += 32) {
      uint32_t o[32];
      if (have_o) {
        tmem_ld32_nw(trow + TL_O_COL + c0, o);
        tmem_wait();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0u;
      }
      if (!row_ok || !alive) continue;
      if (!direct && !(l_sum > 0.f)) continue;      // LSE -inf marks the row empty
      if (on_chip && !direct) {
#pragma unroll
        for (int k = 0; k < 32; k += 4)
          *reinterpret_cast<float4*>(sO + r * 128 + c0 + k) =
              make_float4(__uint_as_float(o[k]) * inv, __uint_as_float(o[k + 1]) * inv,
                          __uint_as_float(o[k + 2]) * inv, __uint_as_float(o[k + 3]) * inv);
      } else if (direct) {
        T* dst = reinterpret_cast<T*>(p.out) + (int64_t)qi * p.out_row_stride + (int64_t)head * 128 + c0;
#pragma unroll
        for (int k = 0; k < 32; k += 8) {
          uint32_t w4[4];
#pragma unroll
          for (int u = 0; u < 4; ++u)
            w4[u] = pack2<T>(__uint_as_float(o[k + 2 * u]) * inv, __uint_as_float(o[k + 2 * u + 1]) * inv);
          *reinterpret_cast<int4*>(dst + k) = make_int4(w4[0], w4[1], w4[2], w4[3]);
        }
      } else {
#pragma unroll
        for (int k = 0; k < 32; k += 8) {
          uint32_t w4[4];
#pragma unroll
          for (int u = 0; u < 4; ++u)
            w4[u] = pack2<T>(__uint_as_float(o[k + 2 * u]) * inv, __uint_as_float(o[k + 2 * u + 1]) * inv);
          *reinterpret_cast<int4*>(prow_o + c0 + k) = make_int4(w4[0], w4[1], w4[2], w4[3]);
        }
      }
    }
    if (tid == 0) tstamp(p, 5);
    if (on_chip && !direct) {
      if (row_ok) sL[r] = alive ? lse2 : -INFINITY;
    } else if (row_ok && alive) {
      if (direct) {
        if (p.lse && !(p.debug & 4)) p.lse[(int64_t)qi * p.hq + head] = lse2 * kLn2;
      } else {
        p.part_lse[((int64_t)(part_base + kidx) * p.hkv + kvh) * M + r] = lse2;
      }
    }
  }
    }
  // ---------------- on-chip merge of a cluster's pieces ----------------
  // Every CTA of the cluster gets here (all waits above are bounded), so the two
  // cluster barriers cannot wait for a CTA that left.
  if (on_chip && t_npieces > 1) {
    cluster_sync();                                 // the cluster's partial rows are written
    const float* sO = reinterpret_cast<const float*>(sStage);
    const float* sL = reinterpret_cast<const float*>(sQ);
    const int cs = p.cluster, rank = (int)cluster_rank();
    const int per = (rows + cs - 1) / cs, r0 = rank * per, r1 = min(rows, r0 + per);
    for (int idx = tid; idx < (r1 - r0) * 32; idx += 192) {
      const int rr = r0 + (idx >> 5), d4 = idx & 31;
      float l[16];
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        l[j] = j < cs ? ld_peer(map_peer(smem_u32(sL + rr), j)) : -INFINITY;
        mx = fmaxf(mx, l[j]);
      }
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      float ws = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if (!(l[j] > -INFINITY)) continue;
        const float w = ex2(l[j] - mx);
        const float4 x = ld_peer4(map_peer(smem_u32(sO + rr * 128 + 4 * d4), j));
        ws += w;
        acc.x += w * x.x;
        acc.y += w * x.y;
        acc.z += w * x.z;
        acc.w += w * x.w;
      }
      const float iw = ws > 0.f ? 1.f / ws : 0.f;
      const int qo = q_begin + rr / p.g, hh = kvh * p.g + rr % p.g;
      T* dst = reinterpret_cast<T*>(p.out) + (int64_t)qo * p.out_row_stride + (int64_t)hh * 128 +
               4 * d4;
      *reinterpret_cast<uint2*>(dst) =
          make_uint2(pack2<T>(acc.x * iw, acc.y * iw), pack2<T>(acc.z * iw, acc.w * iw));
      if (d4 == 0 && p.lse && !(p.debug & 4))
        p.lse[(int64_t)qo * p.hq + hh] = ws > 0.f ? (mx + log2f(ws)) * kLn2 : -INFINITY;
    }
    cluster_sync();                                 // peers finished reading this CTA
  }
  // ---------------- teardown ----------------
  tc_fence_before();
  __syncthreads();
  if (*abort_flag && tid == 160) {
    // copies this CTA issued: let the last NS chunks' loads land before exit
    const int n_iss = *issued;
    for (int c = max(0, n_iss - NS); c < n_iss; ++c) {
      mbar_wait(kfull + c % NS, (c / NS) & 1);
      mbar_wait(vfull + c % NS, (c / NS) & 1);
    }
  }
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "n"(TL_TMEM_COLS)
                 : "memory");
  }
}

// LSE merge of the tiles with several pieces: a grid-stride loop over
// (KV head, tile, row), one warp per row; rows of one-piece tiles (written
// directly by the tile kernel) are skipped.
template <typename T, int M>
__global__ void __launch_bounds__(128) tile_merge_kernel(TileParams p) {
  pdl_wait();                                        // the tile kernel's partial rows
  const int32_t* hdr = p.plan;
  const int n_tiles = __ldg(hdr + 0);
  const int4* tiles = reinterpret_cast<const int4*>(hdr + __ldg(hdr + 4));
  const int g = p.g;
  const int64_t n_rows = (int64_t)p.hkv * n_tiles * M;
  const int64_t warps = (int64_t)gridDim.x * 4;
  for (int64_t w = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5); w < n_rows; w += warps) {
    const int rr = (int)(w % M);
    const int tile = (int)((w / M) % n_tiles);
    const int kvh = (int)(w / ((int64_t)M * n_tiles));
    const int4 t0 = __ldg(tiles + 2 * tile), t1 = __ldg(tiles + 2 * tile + 1);
    const int np = t0.w, part_base = t1.x;
    if (np <= 1 || rr >= min(t0.y * g, M)) continue;
    if (part_base < 0 || part_base + np > p.max_part_pieces) {
      if ((threadIdx.x & 31) == 0) flag_range_error();
      continue;
    }
    const int qr = t0.x + rr / g, hd = kvh * g + rr % g;
    if (np <= 8)          // two groups of 16 lanes (8 dims each): <= 8 pieces per step
      merge_row_warp<T, 2>(p, part_base, np, kvh, M, rr, qr, hd);
    else if (np <= 16)
      merge_row_warp<T, 4>(p, part_base, np, kvh, M, rr, qr, hd);
    else
      merge_row_warp<T, 8>(p, part_base, np, kvh, M, rr, qr, hd);
  }
}

template <typename T, int M>
int launch_tiles(TileParams p, const CUtensorMap& map, int max_pieces, int merge,
                 cudaStream_t st) {
  const size_t smem = TileShape<M>::smem();
  static bool set = false;
  if (!set) {
    BE_CUDA_CHECK(cudaFuncSetAttribute(attn_tile_kernel<T, M>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    // clusters of up to 16 CTAs (beyond the portable 8)
    BE_CUDA_CHECK(cudaFuncSetAttribute(attn_tile_kernel<T, M>,
                                       cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    set = true;
  }
  if (p.cluster > 1) {
    p.merge_next = 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(max_pieces, p.hkv);
    cfg.blockDim = dim3(192);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = p.cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    BE_CUDA_CHECK(cudaLaunchKernelEx(&cfg, attn_tile_kernel<T, M>, map, p));
    return BE_OK;
  }
  p.merge_next = merge && p.max_part_pieces > 0;
  BE_CUDA_CHECK(launch_pdl(attn_tile_kernel<T, M>, dim3(max_pieces, p.hkv), 192, smem, st, map, p));
  if (p.merge_next) {
    const int64_t warps = (int64_t)p.hkv * p.max_tiles * M;
    const int grid = (int)std::min<int64_t>((warps + 3) / 4, 148 * 8);
    BE_CUDA_CHECK(launch_pdl(tile_merge_kernel<T, M>, dim3(grid), 128, 0, st, p));
  }
  return BE_OK;
}

}  // namespace be

extern "C" int be_attn_tiles_run(const int32_t* plan_dev, int max_pieces, int max_tiles,
                                 int max_part_pieces, int tile_rows, int page_size, const void* q,
                                 int64_t q_row_stride, const void* paged_kv_cache, int num_pages,
                                 int num_qo_heads, int num_kv_heads, int head_dim, int dtype,
                                 float sm_scale, void* out, int64_t out_row_stride, float* lse,
                                 void* part_o, float* part_lse, int cluster, int plan_early,
                                 void* stream) {
  using namespace be;
  if (!plan_dev || !q || !paged_kv_cache || !out) {
    set_error("be_attn_tiles_run: null pointer");
    return BE_EINVAL;
  }
  if (dtype != BE_BF16 && dtype != BE_F16) {
    set_error("be_attn_tiles_run: 2-byte pools only (bf16 / f16)");
    return BE_ENOTSUP;
  }
  if (head_dim != 128 || page_size != 16 || num_kv_heads < 1 || num_kv_heads > 65535 ||
      num_qo_heads % num_kv_heads || (tile_rows != 64 && tile_rows != 128)) {
    set_error("be_attn_tiles_run: needs head_dim 128, page size 16, tile_rows 64 or 128 "
              "(got D %d, page %d, rows %d)", head_dim, page_size, tile_rows);
    return BE_ENOTSUP;
  }
  if (cluster < 0 || cluster > 16 || (cluster > 1 && max_pieces % cluster)) {
    set_error("be_attn_tiles_run: cluster %d must be 0..16 and divide max_pieces %d", cluster,
              max_pieces);
    return BE_EINVAL;
  }
  if (max_pieces < 0 || max_tiles < 0 || max_part_pieces < 0) {
    set_error("be_attn_tiles_run: negative capacity");
    return BE_EINVAL;
  }
  if (max_part_pieces > 0 && (!part_o || !part_lse)) {
    set_error("be_attn_tiles_run: partial rows need part_o and part_lse");
    return BE_EINVAL;
  }
  if (((uintptr_t)q | (uintptr_t)paged_kv_cache | (uintptr_t)out) % 16 || q_row_stride % 8 ||
      out_row_stride % 8) {
    set_error("be_attn_tiles_run: q, out and the pool must be 16-byte aligned (row strides %% 8)");
    return BE_EINVAL;
  }
  if (max_pieces == 0) return BE_OK;
  CUtensorMap map;
  int rc = get_pool_map(paged_kv_cache, num_pages, page_size, num_kv_heads, head_dim, dtype, &map);
  if (rc != BE_OK) return rc;
  TileParams p;
  p.plan = plan_dev;
  p.q = (const char*)q;
  p.q_row_stride = q_row_stride;
  p.num_pages = num_pages;
  p.hq = num_qo_heads;
  p.hkv = num_kv_heads;
  p.g = num_qo_heads / num_kv_heads;
  p.scale_log2 = sm_scale * kLog2e;
  p.out = (char*)out;
  p.out_row_stride = out_row_stride;
  p.lse = lse;
  p.part_o = part_o;
  p.part_lse = part_lse;
  p.max_part_pieces = max_part_pieces;
  p.max_tiles = max_tiles;
  p.plan_early = plan_early;
  p.cluster = cluster > 1 ? cluster : 0;
  const char* dbg = getenv("BE_ATTN_DEBUG");
  p.debug = dbg ? atoi(dbg) : 0;
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == BE_BF16)
    return tile_rows == 64 ? launch_tiles<__nv_bfloat16, 64>(p, map, max_pieces, 1, st)
                           : launch_tiles<__nv_bfloat16, 128>(p, map, max_pieces, 1, st);
  return tile_rows == 64 ? launch_tiles<__half, 64>(p, map, max_pieces, 1, st)
                         : launch_tiles<__half, 128>(p, map, max_pieces, 1, st);
}
