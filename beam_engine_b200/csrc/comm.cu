// Tensor-parallel all-reduce over peer memory, fused with the residual add and
// the RMSNorm that follow it in the decoder layer.
//
// The row-parallel projections (o_proj, down_proj) end in an all-reduce of a
// [rows, hidden] partial, and the layer continues with residual += sum;
// h = rmsnorm(residual) * w.  For decode (128 rows x 4096 = 1 MiB) a ring
// all-reduce is latency-bound, so each rank instead:
//   1. has its GEMM write the partial straight into its own slot of a buffer
//      the other ranks have mapped (CUDA IPC, one process per GPU);
//   2. per CTA (one CTA per row, grid-stride beyond the flag capacity): thread
//      p signals rank p with a per-CTA counter (a relaxed system-scope store to
//      the peer's flag array) and waits until rank p has signalled the same
//      count (ld.acquire.sys, bounded by %globaltimer: on expiry
//      BE_EDEVICE_TIMEOUT is recorded and the CTA returns);
//   3. reads the row from every rank's slot (16-byte loads over NVLink, all
//      ranks' loads in flight together, L1 bypassed), sums in rank order so
//      every rank computes identical bits, in fp32, rounds to the storage
//      type, adds it to the residual, and writes the normalised row -- the
//      add_rmsnorm kernel's arithmetic.
// Consecutive calls alternate between two slots: a rank can only write a slot
// again after the barrier of the call in between, which every rank reaches
// after finishing its reads of that slot -- so no closing barrier is needed.
// No TMA, no multicast: peers' memory is only touched by plain loads/stores.
#include "common.cuh"

#include <cstring>
#include <vector>

namespace be {

constexpr int COMM_MAX_RANKS = 8;
constexpr uint64_t kCommWaitNs = 2000000000ull;   // 2 s

struct CommArgs {
  uint32_t* flags_out[COMM_MAX_RANKS];  // every rank's incoming-flag array
  uint32_t* flags_in;                   // this rank's: [cta][src rank]
  uint32_t* counter;                    // this rank's per-CTA call counter
  const char* slot[COMM_MAX_RANKS];     // every rank's slot of this call
  int rank, world, max_ctas;
};

__device__ __forceinline__ uint64_t comm_gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Barrier of CTA `cta` across ranks; false if it timed out.  Thread p < world
// signals rank p and waits for rank p's signal, so the peers are served in
// parallel.  The signal is a relaxed store with no fence: the data it
// announces (this rank's slot) was written by kernels that completed before
// this one started, and peers read it from this GPU's L2 over NVLink.  (A
// release fence at system scope cost ~10 us per call here.)  The wait is an
// acquire load, so this thread's later reads stay behind it; the block
// barrier after it orders the other threads' reads.
__device__ bool comm_barrier(const CommArgs& a, int cta, uint32_t* epoch_out = nullptr) {
  __shared__ uint32_t epoch;
  __shared__ int ok;
  const int t = threadIdx.x;
  if (t == 0) {
    epoch = a.counter[cta] + 1;
    ok = 1;
  }
  __syncthreads();
  const uint32_t e = epoch;
  if (epoch_out) *epoch_out = e;
  if (t < a.world) {
    st_relaxed_sys(a.flags_out[t] + (size_t)cta * COMM_MAX_RANKS + a.rank, e);
    const uint32_t* f = a.flags_in + (size_t)cta * COMM_MAX_RANKS + t;
    const uint64_t t0 = comm_gtimer();
    int polls = 0;
    while ((int32_t)(ld_acquire_sys(f) - e) < 0) {   // monotonic: a peer may be ahead
      if (++polls == 64) {
        polls = 0;
        if (comm_gtimer() - t0 > kCommWaitNs) {
          atomicCAS(&g_device_status, 0, BE_EDEVICE_TIMEOUT);
          ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  if (t == 0) a.counter[cta] = e;
  return ok != 0;
}

template <typename T>
__device__ __forceinline__ void unpack16(const int4& raw, float* out) {
  if constexpr (sizeof(T) == 2) {
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = to_f(e[i]);
  } else {
    out[0] = __int_as_float(raw.x);
    out[1] = __int_as_float(raw.y);
    out[2] = __int_as_float(raw.z);
    out[3] = __int_as_float(raw.w);
  }
}
template <typename T>
__device__ __forceinline__ void load16(const T* p, float* out) {
  const int4 raw = *reinterpret_cast<const int4*>(p);
  if constexpr (sizeof(T) == 2) {
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = to_f(e[i]);
  } else {
    out[0] = __int_as_float(raw.x);
    out[1] = __int_as_float(raw.y);
    out[2] = __int_as_float(raw.z);
    out[3] = __int_as_float(raw.w);
  }
}
template <typename T>
__device__ __forceinline__ void store16(T* p, const float* v) {
  int4 raw;
  if constexpr (sizeof(T) == 2) {
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) e[i] = from_f<T>(v[i]);
  } else {
    raw = make_int4(__float_as_int(v[0]), __float_as_int(v[1]), __float_as_int(v[2]),
                    __float_as_int(v[3]));
  }
  *reinterpret_cast<int4*>(p) = raw;
}

constexpr int COMM_THREADS = 512;
constexpr int COMM_NV = 4;   // 16-byte vectors per thread: hidden <= 512 x 4 x (16 / sizeof(T))

// One CTA per row (grid-stride), one 16-byte vector of the row per thread and
// pass (blockDim = hidden / vector width, up to 512 threads).  Every rank's
// vector is loaded before any is summed, so the row costs one NVLink round
// trip; sums in rank order (identical bits on every rank).  With residual:
// residual += round_T(sum); out = w * round_T(residual * rsqrt(mean(residual^2)
// + eps)).  Without it: out = round_T(sum).
template <typename T>
__global__ void __launch_bounds__(COMM_THREADS) allreduce_rmsnorm_kernel(
    CommArgs a, T* __restrict__ residual, const T* __restrict__ w, T* __restrict__ out, int rows,
    int H, float eps) {
  constexpr int V = 16 / sizeof(T);
  const int cta = blockIdx.x;
  pdl_wait();                      // the partials come from the kernel before this one
  if (!comm_barrier(a, cta)) return;
  __shared__ float red[32];
  for (int row = cta; row < rows; row += gridDim.x) {
    float cache[COMM_NV][V];
    float ss = 0.f;
    const int64_t base = (int64_t)row * H;
#pragma unroll
    for (int nv = 0; nv < COMM_NV; ++nv) {
      const int c = (threadIdx.x + nv * blockDim.x) * V;
      if (c >= H) break;
      int4 raw[COMM_MAX_RANKS];
#pragma unroll
      for (int p = 0; p < COMM_MAX_RANKS; ++p)   // L1-bypassing loads, all in flight
        if (p < a.world)
          raw[p] = __ldcv(reinterpret_cast<const int4*>(
              reinterpret_cast<const T*>(a.slot[p]) + base + c));
      float s[V];
      unpack16<T>(raw[0], s);
#pragma unroll
      for (int p = 1; p < COMM_MAX_RANKS; ++p) {
        if (p >= a.world) break;
        float t[V];
        unpack16<T>(raw[p], t);
#pragma unroll
        for (int i = 0; i < V; ++i) s[i] += t[i];
      }
      if (residual) {
        float x[V];
        load16(residual + base + c, x);
#pragma unroll
        for (int i = 0; i < V; ++i) x[i] = to_f(from_f<T>(x[i] + to_f(from_f<T>(s[i]))));
        store16(residual + base + c, x);
#pragma unroll
        for (int i = 0; i < V; ++i) {
          ss += x[i] * x[i];
          cache[nv][i] = x[i];
        }
      } else {
        store16(out + base + c, s);
      }
    }
    if (!residual) continue;
#pragma unroll
    for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
      float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
      for (int off = 16; off; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float inv = rsqrtf(red[0] / (float)H + eps);
#pragma unroll
    for (int nv = 0; nv < COMM_NV; ++nv) {
      const int c = (threadIdx.x + nv * blockDim.x) * V;
      if (c >= H) break;
      float wv[V], r[V];
      load16(w + c, wv);
#pragma unroll
      for (int i = 0; i < V; ++i) r[i] = wv[i] * to_f(from_f<T>(cache[nv][i] * inv));
      store16(out + base + c, r);
    }
    __syncthreads();   // red[] is reused by the next row
  }
}


// Two-shot form for many ranks (one-shot reads world - 1 full partials per
// rank over NVLink: 7 MiB per call at 8 ranks).  Row r belongs to rank
// r % world: its owner sums the ranks' partial rows, adds the residual and
// stores the new residual row over its own partial row (only the owner reads
// that row of its slot), then signals every rank; the other ranks wait for the
// owner's signal and copy the row from its slot.  Every rank then applies the
// RMSNorm to its copy: the same bits as the one-shot kernel, with about
// 2 x (world - 1) / world rows read per rank instead of world - 1.
// Row flags: uint32 [max_ctas] after the barrier flags and counters.
__device__ __forceinline__ uint32_t* comm_row_flags(uint32_t* flags, int max_ctas) {
  return flags + (size_t)max_ctas * COMM_MAX_RANKS + max_ctas;
}

template <typename T>
__global__ void __launch_bounds__(COMM_THREADS) allreduce_rmsnorm_2shot_kernel(
    CommArgs a, T* __restrict__ residual, const T* __restrict__ w, T* __restrict__ out, int rows,
    int H, float eps) {
  constexpr int V = 16 / sizeof(T);
  const int row = blockIdx.x;      // rows <= max_ctas: one CTA per row
  pdl_wait();                      // the partials come from the kernel before this one
  uint32_t e = 0;
  if (!comm_barrier(a, row, &e)) return;
  __shared__ float red[32];
  __shared__ int ok;
  const int owner = row % a.world;
  const int64_t base = (int64_t)row * H;
  float cache[COMM_NV][V];
  float ss = 0.f;
  if (owner == a.rank) {
    T* mine = reinterpret_cast<T*>(const_cast<char*>(a.slot[a.rank]));
#pragma unroll
    for (int nv = 0; nv < COMM_NV; ++nv) {
      const int c = (threadIdx.x + nv * blockDim.x) * V;
      if (c >= H) break;
      int4 raw[COMM_MAX_RANKS];
#pragma unroll
      for (int p = 0; p < COMM_MAX_RANKS; ++p)
        if (p < a.world)
          raw[p] = __ldcv(reinterpret_cast<const int4*>(
              reinterpret_cast<const T*>(a.slot[p]) + base + c));
      float sum[V];
      unpack16<T>(raw[0], sum);
#pragma unroll
      for (int p = 1; p < COMM_MAX_RANKS; ++p) {
        if (p >= a.world) break;
        float t[V];
        unpack16<T>(raw[p], t);
#pragma unroll
        for (int i = 0; i < V; ++i) sum[i] += t[i];
      }
      float x[V];
      load16(residual + base + c, x);
#pragma unroll
      for (int i = 0; i < V; ++i) x[i] = to_f(from_f<T>(x[i] + to_f(from_f<T>(sum[i]))));
      store16(residual + base + c, x);
      store16(mine + base + c, x);            // the new residual row, for the other ranks
#pragma unroll
      for (int i = 0; i < V; ++i) {
        ss += x[i] * x[i];
        cache[nv][i] = x[i];
      }
    }
    asm volatile("fence.acq_rel.gpu;" ::: "memory");   // the row is in this GPU's L2
    __syncthreads();
    if (threadIdx.x < a.world && threadIdx.x != a.rank)
      st_relaxed_sys(comm_row_flags(a.flags_out[threadIdx.x], a.max_ctas) + row, e);
  } else {
    if (threadIdx.x == 0) {
      ok = 1;
      const uint32_t* f = comm_row_flags(a.flags_in, a.max_ctas) + row;
      const uint64_t t0 = comm_gtimer();
      int polls = 0;
      while ((int32_t)(ld_acquire_sys(f) - e) < 0) {
        if (++polls == 64) {
          polls = 0;
          if (comm_gtimer() - t0 > kCommWaitNs) {
            atomicCAS(&g_device_status, 0, BE_EDEVICE_TIMEOUT);
            ok = 0;
            break;
          }
        }
      }
    }
    __syncthreads();
    if (!ok) return;
    const T* src = reinterpret_cast<const T*>(a.slot[owner]);
#pragma unroll
    for (int nv = 0; nv < COMM_NV; ++nv) {
      const int c = (threadIdx.x + nv * blockDim.x) * V;
      if (c >= H) break;
      float x[V];
      unpack16<T>(__ldcv(reinterpret_cast<const int4*>(src + base + c)), x);
      store16(residual + base + c, x);
#pragma unroll
      for (int i = 0; i < V; ++i) {
        ss += x[i] * x[i];
        cache[nv][i] = x[i];
      }
    }
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int off = 16; off; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)H + eps);
#pragma unroll
  for (int nv = 0; nv < COMM_NV; ++nv) {
    const int c = (threadIdx.x + nv * blockDim.x) * V;
    if (c >= H) break;
    float wv[V], r[V];
    load16(w + c, wv);
#pragma unroll
    for (int i = 0; i < V; ++i) r[i] = wv[i] * to_f(from_f<T>(cache[nv][i] * inv));
    store16(out + base + c, r);
  }
}

// Vocabulary-parallel scoring exchange: every rank's be_logsoftmax_topk wrote
// its slice's top k (value desc, global id asc), row max and sum of
// exponentials into its slot (layout of comm_topk_layout).  One CTA per row:
// the log-sum-exp over the ranks (rank order, identical bits on every rank),
// then every candidate's rank among all ranks' lists by binary search; ranks
// 0..k-1 are written as log-probabilities with their ids.
struct TopkSlot {
  int64_t idx_off, val_off, max_off, sum_off;   // bytes from the slot start
};
__host__ __device__ inline TopkSlot comm_topk_layout(int rows, int k) {
  TopkSlot t;
  t.idx_off = 0;
  t.val_off = (int64_t)rows * k * 8;
  t.max_off = t.val_off + (int64_t)rows * k * 4;
  t.sum_off = t.max_off + (int64_t)rows * 4;
  return t;
}
constexpr int COMM_TOPK_MAX = 64;

__device__ __forceinline__ bool topk_better(float a, int64_t ia, float b, int64_t ib) {
  return a > b || (a == b && ia < ib);
}

__global__ void __launch_bounds__(128) topk_merge_kernel(CommArgs a, int rows, int k,
                                                         float* __restrict__ out_val,
                                                         int64_t* __restrict__ out_idx) {
  const int cta = blockIdx.x;
  pdl_wait();                      // the slices' top-k come from the kernel before this one
  if (!comm_barrier(a, cta)) return;
  __shared__ float sv[COMM_MAX_RANKS * COMM_TOPK_MAX];
  __shared__ int64_t si[COMM_MAX_RANKS * COMM_TOPK_MAX];
  __shared__ float s_lse;
  const TopkSlot L = comm_topk_layout(rows, k);
  const int tot = a.world * k;
  for (int row = cta; row < rows; row += gridDim.x) {
    for (int e = threadIdx.x; e < tot; e += blockDim.x) {
      const int p = e / k, j = e - p * k;
      const char* base = a.slot[p];
      si[e] = __ldcv(reinterpret_cast<const long long*>(base + L.idx_off) + (int64_t)row * k + j);
      sv[e] = __ldcv(reinterpret_cast<const float*>(base + L.val_off) + (int64_t)row * k + j);
    }
    if (threadIdx.x == 0) {
      float m = -INFINITY;
      for (int p = 0; p < a.world; ++p)
        m = fmaxf(m, __ldcv(reinterpret_cast<const float*>(a.slot[p] + L.max_off) + row));
      float s = 0.f;
      for (int p = 0; p < a.world; ++p) {
        const float mp = __ldcv(reinterpret_cast<const float*>(a.slot[p] + L.max_off) + row);
        const float sp = __ldcv(reinterpret_cast<const float*>(a.slot[p] + L.sum_off) + row);
        if (mp > -INFINITY) s += sp * expf(mp - m);
      }
      s_lse = m + logf(s);
    }
    __syncthreads();
    const float lse = s_lse;
    for (int e = threadIdx.x; e < tot; e += blockDim.x) {
      const int p = e / k;
      const float xv = sv[e];
      const int64_t xi = si[e];
      int rank = e - p * k;               // entries of its own list before it
      for (int q = 0; q < a.world && rank < k; ++q) {
        if (q == p) continue;
        int lo = 0, hi = k;
        while (lo < hi) {
          const int mid = (lo + hi) >> 1;
          if (topk_better(sv[q * k + mid], si[q * k + mid], xv, xi)) lo = mid + 1;
          else hi = mid;
        }
        rank += lo;
      }
      if (rank < k) {
        out_val[(int64_t)row * k + rank] = xv - lse;
        out_idx[(int64_t)row * k + rank] = xi;
      }
    }
    __syncthreads();               // sv / si / s_lse are reused by the next row
  }
}
}  // namespace be

using namespace be;

struct be_comm {
  int rank = 0, world = 0, num_slots = 0, max_ctas = 0, device = 0;
  int64_t slot_bytes = 0;
  size_t flags_bytes = 0;       // flags + counters, rounded up to 256
  char* base = nullptr;         // this rank's allocation
  char* peer[COMM_MAX_RANKS] = {};
  bool opened[COMM_MAX_RANKS] = {};
  cudaIpcMemHandle_t own;       // this rank's handle (a peer given it maps to this buffer)
};

static size_t comm_flags_bytes(int max_ctas) {
  // barrier flags [cta][rank], per-CTA counters, two-shot row flags [cta]
  const size_t b = (size_t)max_ctas * COMM_MAX_RANKS * 4 + 2 * (size_t)max_ctas * 4;
  return (b + 255) / 256 * 256;
}

extern "C" int be_comm_create(int world, int rank, int64_t slot_bytes, int num_slots,
                              int max_ctas, void* handle_out, be_comm** out) {
  if (!out || !handle_out || world < 1 || world > COMM_MAX_RANKS || rank < 0 || rank >= world ||
      slot_bytes < 16 || slot_bytes % 16 || num_slots < 1 || max_ctas < 1) {
    set_error("be_comm_create: invalid arguments (world <= %d, 16-byte slots)", COMM_MAX_RANKS);
    return BE_EINVAL;
  }
  auto* c = new be_comm();
  c->rank = rank;
  c->world = world;
  c->num_slots = num_slots;
  c->max_ctas = max_ctas;
  c->slot_bytes = slot_bytes;
  c->flags_bytes = comm_flags_bytes(max_ctas);
  cudaGetDevice(&c->device);
  const size_t total = c->flags_bytes + (size_t)num_slots * slot_bytes;
  cudaError_t e = cudaMalloc(&c->base, total);
  if (e == cudaSuccess) e = cudaMemset(c->base, 0, c->flags_bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&c->own, c->base);
  if (e == cudaSuccess) std::memcpy(handle_out, &c->own, sizeof(c->own));
  if (e != cudaSuccess) {
    set_error("be_comm_create: %s", cudaGetErrorString(e));
    if (c->base) cudaFree(c->base);
    delete c;
    return BE_ECUDA;
  }
  c->peer[rank] = c->base;
  *out = c;
  return BE_OK;
}

extern "C" int be_comm_open(be_comm* c, const void* handles) {
  if (!c || !handles) {
    set_error("be_comm_open: invalid arguments");
    return BE_EINVAL;
  }
  const auto* h = reinterpret_cast<const cudaIpcMemHandle_t*>(handles);
  for (int p = 0; p < c->world; ++p) {
    if (p == c->rank || c->opened[p]) continue;
    if (std::memcmp(&h[p], &c->own, sizeof(c->own)) == 0) {
      c->peer[p] = c->base;   // loopback: this rank's own buffer stands in for rank p
      continue;
    }
    void* ptr = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&ptr, h[p], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      set_error("be_comm_open: rank %d: %s", p, cudaGetErrorString(e));
      return BE_ECUDA;
    }
    c->peer[p] = reinterpret_cast<char*>(ptr);
    c->opened[p] = true;
  }
  return BE_OK;
}

extern "C" void* be_comm_flags(be_comm* c) { return c ? c->base : nullptr; }

extern "C" void* be_comm_slot(be_comm* c, int slot) {
  if (!c || slot < 0 || slot >= c->num_slots) return nullptr;
  return c->base + c->flags_bytes + (size_t)slot * c->slot_bytes;
}

extern "C" int be_comm_close_peers(be_comm* c) {
  if (!c) return BE_OK;
  cudaDeviceSynchronize();
  for (int p = 0; p < c->world; ++p)
    if (c->opened[p]) {
      cudaIpcCloseMemHandle(c->peer[p]);
      c->opened[p] = false;
      c->peer[p] = nullptr;
    }
  return BE_OK;
}

extern "C" int be_comm_destroy(be_comm* c) {
  if (!c) return BE_OK;
  be_comm_close_peers(c);
  if (c->base) cudaFree(c->base);
  delete c;
  return BE_OK;
}

extern "C" int be_comm_allreduce_rmsnorm(be_comm* c, int slot, void* residual, const void* norm_w,
                                         void* out, int rows, int hidden, float eps, int dtype,
                                         void* stream) {
  if (!c || slot < 0 || slot >= c->num_slots || !out || rows < 0 || hidden < 1 ||
      dtype < BE_F32 || dtype > BE_BF16 || (residual && !norm_w)) {
    set_error("be_comm_allreduce_rmsnorm: invalid arguments");
    return BE_EINVAL;
  }
  const int elt = dtype_size(dtype), V = 16 / elt;
  if ((int64_t)rows * hidden * elt > c->slot_bytes || hidden % V || hidden / V > COMM_THREADS * COMM_NV ||
      ((uintptr_t)out | (uintptr_t)residual | (uintptr_t)norm_w) % 16) {
    set_error("be_comm_allreduce_rmsnorm: %d x %d does not fit a %lld-byte slot / 16-byte rows",
              rows, hidden, (long long)c->slot_bytes);
    return BE_EINVAL;
  }
  for (int p = 0; p < c->world; ++p)
    if (!c->peer[p]) {
      set_error("be_comm_allreduce_rmsnorm: rank %d not opened (be_comm_open)", p);
      return BE_EINVAL;
    }
  if (rows == 0) return BE_OK;
  CommArgs a = {};
  for (int p = 0; p < c->world; ++p) {
    a.flags_out[p] = reinterpret_cast<uint32_t*>(c->peer[p]);
    a.slot[p] = c->peer[p] + c->flags_bytes + (size_t)slot * c->slot_bytes;
  }
  a.flags_in = reinterpret_cast<uint32_t*>(c->base);
  a.counter = reinterpret_cast<uint32_t*>(c->base + (size_t)c->max_ctas * COMM_MAX_RANKS * 4);
  a.rank = c->rank;
  a.world = c->world;
  a.max_ctas = c->max_ctas;
  const int grid = std::min(rows, c->max_ctas);
  const int threads = std::min(COMM_THREADS, std::max(32, (hidden / V + 31) / 32 * 32));
  cudaStream_t st = (cudaStream_t)stream;
  // two-shot from BE_COMM_TWO_SHOT_WORLD ranks on (default 4; 0 = never)
  static const int two_shot_world = [] {
    const char* v = getenv("BE_COMM_TWO_SHOT_WORLD");
    return v ? atoi(v) : 4;
  }();
  if (residual && two_shot_world > 0 && c->world >= two_shot_world && rows <= c->max_ctas) {
    switch (dtype) {
      case BE_BF16:
        BE_CUDA_CHECK(launch_pdl(allreduce_rmsnorm_2shot_kernel<__nv_bfloat16>, rows, threads, 0,
                                 st, a, (__nv_bfloat16*)residual, (const __nv_bfloat16*)norm_w,
                                 (__nv_bfloat16*)out, rows, hidden, eps));
        break;
      case BE_F16:
        BE_CUDA_CHECK(launch_pdl(allreduce_rmsnorm_2shot_kernel<__half>, rows, threads, 0, st, a,
                                 (__half*)residual, (const __half*)norm_w, (__half*)out, rows,
                                 hidden, eps));
        break;
      default:
        BE_CUDA_CHECK(launch_pdl(allreduce_rmsnorm_2shot_kernel<float>, rows, threads, 0, st, a,
                                 (float*)residual, (const float*)norm_w, (float*)out, rows, hidden,
                                 eps));
    }
    BE_LAUNCH_CHECK();
    return BE_OK;
  }
  switch (dtype) {
    case BE_BF16:
      BE_CUDA_CHECK(launch_pdl(allreduce_rmsnorm_kernel<__nv_bfloat16>, grid, threads, 0, st,
          a, (__nv_bfloat16*)residual, (const __nv_bfloat16*)norm_w, (__nv_bfloat16*)out, rows,
          hidden, eps));
      break;
    case BE_F16:
      BE_CUDA_CHECK(launch_pdl(allreduce_rmsnorm_kernel<__half>, grid, threads, 0, st,
          a, (__half*)residual, (const __half*)norm_w, (__half*)out, rows, hidden, eps));
      break;
    default:
      BE_CUDA_CHECK(launch_pdl(allreduce_rmsnorm_kernel<float>, grid, threads, 0, st,
          a, (float*)residual, (const float*)norm_w, (float*)out, rows, hidden, eps));
  }
  BE_LAUNCH_CHECK();
  return BE_OK;
}

extern "C" int be_comm_topk_layout(int rows, int k, int64_t* offsets) {
  if (rows < 0 || k < 1 || !offsets) {
    set_error("be_comm_topk_layout: invalid arguments");
    return BE_EINVAL;
  }
  const TopkSlot t = comm_topk_layout(rows, k);
  offsets[0] = t.idx_off;
  offsets[1] = t.val_off;
  offsets[2] = t.max_off;
  offsets[3] = t.sum_off;
  return BE_OK;
}

extern "C" int be_comm_topk_merge(be_comm* c, int slot, int rows, int k, float* out_val,
                                  int64_t* out_idx, void* stream) {
  if (!c || slot < 0 || slot >= c->num_slots || rows < 0 || k < 1 || k > COMM_TOPK_MAX ||
      !out_val || !out_idx || c->world * k > COMM_MAX_RANKS * COMM_TOPK_MAX) {
    set_error("be_comm_topk_merge: invalid arguments (k <= %d)", COMM_TOPK_MAX);
    return BE_EINVAL;
  }
  const TopkSlot t = comm_topk_layout(rows, k);
  if (t.sum_off + (int64_t)rows * 4 > c->slot_bytes) {
    set_error("be_comm_topk_merge: %d rows x top-%d do not fit a %lld-byte slot", rows, k,
              (long long)c->slot_bytes);
    return BE_EINVAL;
  }
  for (int p = 0; p < c->world; ++p)
    if (!c->peer[p]) {
      set_error("be_comm_topk_merge: rank %d not opened (be_comm_open)", p);
      return BE_EINVAL;
    }
  if (rows == 0) return BE_OK;
  CommArgs a = {};
  for (int p = 0; p < c->world; ++p) {
    a.flags_out[p] = reinterpret_cast<uint32_t*>(c->peer[p]);
    a.slot[p] = c->peer[p] + c->flags_bytes + (size_t)slot * c->slot_bytes;
  }
  a.flags_in = reinterpret_cast<uint32_t*>(c->base);
  a.counter = reinterpret_cast<uint32_t*>(c->base + (size_t)c->max_ctas * COMM_MAX_RANKS * 4);
  a.rank = c->rank;
  a.world = c->world;
  a.max_ctas = c->max_ctas;
  const int grid = std::min(rows, c->max_ctas);
  BE_CUDA_CHECK(launch_pdl(topk_merge_kernel, grid, 128, 0, (cudaStream_t)stream, a, rows, k,
                           out_val, out_idx));
  BE_LAUNCH_CHECK();
  return BE_OK;
}
