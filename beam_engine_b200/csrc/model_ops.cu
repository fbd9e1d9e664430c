// Decoder-layer kernels around the attention path (the reference runs these as
// separate PyTorch ops, modeling_llama.py:68-173, 428-562):
//   * add_rmsnorm      residual += delta; out = w * rmsnorm(residual)   (one pass)
//   * rope_append      RoPE on q and k inside the fused QKV output, k and v
//                      written straight into their KV pages (replaces RoPE +
//                      append_paged_kv_cache: one launch, no K/V round trip)
//   * silu_mul         act = silu(gate) * up on the fused gate/up output
// All are HBM-bound row kernels with 16-byte vector loads.
#include "common.cuh"

namespace be {

template <typename T>
struct Vec8 {  // 8 elements = 16 bytes for 2-byte types
  static constexpr int N = 16 / sizeof(T);
};

template <typename T, int N>
__device__ __forceinline__ void load_vec(const T* p, float* out) {
  if constexpr (sizeof(T) == 2) {
    int4 raw = *reinterpret_cast<const int4*>(p);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = to_f(e[i]);
  } else {
    float4 raw = *reinterpret_cast<const float4*>(p);
    out[0] = raw.x; out[1] = raw.y; out[2] = raw.z; out[3] = raw.w;
  }
}
template <typename T, int N>
__device__ __forceinline__ void store_vec(T* p, const float* v) {
  if constexpr (sizeof(T) == 2) {
    int4 raw;
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) e[i] = from_f<T>(v[i]);
    *reinterpret_cast<int4*>(p) = raw;
  } else {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
}

// One CTA per row.  residual (in/out) [rows][H]; delta may be null.
// out = w * round_T(x * rsqrt(mean(x^2) + eps)), x = round_T(residual + delta)
// (the reference: hidden in fp32, normalised, cast back, times the weight).
template <typename T>
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(T* __restrict__ residual,
                                                          const T* __restrict__ delta,
                                                          const T* __restrict__ w,
                                                          T* __restrict__ out, int H, float eps) {
  pdl_wait();   // inputs come from the previous kernel (launched with launch_pdl)
  constexpr int V = 16 / sizeof(T);
  const int row = blockIdx.x;
  T* x = residual + (int64_t)row * H;
  const T* dl = delta ? delta + (int64_t)row * H : nullptr;
  T* o = out + (int64_t)row * H;
  float ss = 0.f;
  // H <= 256 threads * 8 vectors * V elements (16384 for 2-byte types); the
  // loops are unrolled so the row cache stays in registers
  float cache[8][V];
#pragma unroll
  for (int nv = 0; nv < 8; ++nv) {
    const int c = (threadIdx.x + nv * blockDim.x) * V;
    if (c >= H) break;
    float a[V];
    load_vec<T, V>(x + c, a);
    if (dl) {
      float b[V];
      load_vec<T, V>(dl + c, b);
#pragma unroll
      for (int i = 0; i < V; ++i) a[i] = to_f(from_f<T>(a[i] + b[i]));
      store_vec<T, V>(x + c, a);
    }
#pragma unroll
    for (int i = 0; i < V; ++i) {
      ss += a[i] * a[i];
      cache[nv][i] = a[i];
    }
  }
  __shared__ float red[32];
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
  for (int nv = 0; nv < 8; ++nv) {
    const int c = (threadIdx.x + nv * blockDim.x) * V;
    if (c >= H) break;
    float wv[V], r[V];
    load_vec<T, V>(w + c, wv);
#pragma unroll
    for (int i = 0; i < V; ++i) r[i] = wv[i] * to_f(from_f<T>(cache[nv][i] * inv));
    store_vec<T, V>(o + c, r);
  }
}

// RoPE (HF rotate_half convention) on q and k of the fused QKV rows, then k and
// v appended into the pages.  One warp per (row, head) of q/k and per row of v
// heads; pairs (d, d + D/2) rotate by angle pos * inv_freq[d].
template <typename T>
__global__ void __launch_bounds__(256) rope_append_kernel(
    T* __restrict__ qkv, int64_t row_stride, int n, int hq, int hkv, int D,
    const int32_t* __restrict__ positions, const float* __restrict__ inv_freq,
    T* __restrict__ pool, int num_pages, int page_size, const int32_t* __restrict__ write_page,
    const int32_t* __restrict__ write_pos, int write_rope_k_in_place) {
  pdl_wait();
  pdl_trigger();   // the attention launch after this one prepares (plan reads, TMEM) meanwhile
  const int warps_per_row = hq + 2 * hkv;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= n * warps_per_row) return;
  const int row = gw / warps_per_row, h = gw % warps_per_row;
  T* src = qkv + row * row_stride + (int64_t)h * D;
  const int half = D / 2;
  if (h < hq + hkv) {  // q or k head: rotate
    const float pos = (float)positions[row];
    T* dst = src;
    bool to_pool = false;
    if (h >= hq) {  // k head -> page
      const int page = write_page[row], slot = write_pos[row];
      if (page < 0 || page >= num_pages || slot < 0 || slot >= page_size) {
        if (lane == 0) flag_range_error();
        return;
      }
      dst = pool + (((int64_t)page * 2 + 0) * page_size + slot) * hkv * D + (int64_t)(h - hq) * D;
      to_pool = true;
    }
    for (int d = lane; d < half; d += 32) {
      const float ang = pos * inv_freq[d];
      float s, c;
      sincosf(ang, &s, &c);
      const float x1 = to_f(src[d]), x2 = to_f(src[d + half]);
      const T y1 = from_f<T>(x1 * c - x2 * s);
      const T y2 = from_f<T>(x2 * c + x1 * s);
      dst[d] = y1;
      dst[d + half] = y2;
      if (to_pool && write_rope_k_in_place) {
        src[d] = y1;
        src[d + half] = y2;
      }
    }
  } else {  // v head -> page
    const int page = write_page[row], slot = write_pos[row];
    if (page < 0 || page >= num_pages || slot < 0 || slot >= page_size) {
      if (lane == 0) flag_range_error();
      return;
    }
    T* dst = pool + (((int64_t)page * 2 + 1) * page_size + slot) * hkv * D +
             (int64_t)(h - hq - hkv) * D;
    for (int d = lane; d < D; d += 32) dst[d] = src[d];
  }
}

// The same RoPE + append with one CTA per row: the row's cos / sin are computed
// once into shared memory (rope_append_kernel computes them again for every
// head), and every q / k / v access is a 16-byte vector.  Arithmetic per
// element is the same as rope_append_kernel's.  Needs D / 2 a multiple of the
// vector width, D / 2 <= 256, and 16-byte aligned rows and pool.
template <typename T>
__global__ void __launch_bounds__(256) rope_append_rows_kernel(
    T* __restrict__ qkv, int64_t row_stride, int n, int hq, int hkv, int D,
    const int32_t* __restrict__ positions, const float* __restrict__ inv_freq,
    T* __restrict__ pool, int num_pages, int page_size, const int32_t* __restrict__ write_page,
    const int32_t* __restrict__ write_pos, int write_rope_k_in_place) {
  constexpr int V = 16 / sizeof(T);
  __shared__ float cs[256], sn[256];
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x, half = D / 2;
  const float pos = (float)positions[row];
  for (int d = threadIdx.x; d < half; d += blockDim.x) {
    float s, c;
    sincosf(pos * inv_freq[d], &s, &c);
    cs[d] = c;
    sn[d] = s;
  }
  const int page = write_page[row], slot = write_pos[row];
  const bool kv_ok = page >= 0 && page < num_pages && slot >= 0 && slot < page_size;
  if (!kv_ok && threadIdx.x == 0) flag_range_error();
  __syncthreads();
  T* src_row = qkv + row * row_stride;
  const int64_t kdst = ((int64_t)page * 2 * page_size + slot) * hkv * D;      // K half of the page
  const int64_t vdst = (((int64_t)page * 2 + 1) * page_size + slot) * hkv * D;
  const int nvec = half / V;
  const int rot = (kv_ok ? hq + hkv : hq) * nvec;
  for (int i = threadIdx.x; i < rot; i += blockDim.x) {
    const int h = i / nvec, d0 = (i - h * nvec) * V;
    T* src = src_row + (int64_t)h * D;
    float x1[V], x2[V], y1[V], y2[V];
    load_vec<T, V>(src + d0, x1);
    load_vec<T, V>(src + d0 + half, x2);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const float c = cs[d0 + j], s = sn[d0 + j];
      y1[j] = x1[j] * c - x2[j] * s;
      y2[j] = x2[j] * c + x1[j] * s;
    }
    if (h < hq) {
      store_vec<T, V>(src + d0, y1);
      store_vec<T, V>(src + d0 + half, y2);
    } else {
      T* dst = pool + kdst + (int64_t)(h - hq) * D;
      store_vec<T, V>(dst + d0, y1);
      store_vec<T, V>(dst + d0 + half, y2);
      if (write_rope_k_in_place) {
        store_vec<T, V>(src + d0, y1);
        store_vec<T, V>(src + d0 + half, y2);
      }
    }
  }
  if (!kv_ok) return;
  const int vv = hkv * D / V;   // v heads: a straight 16-byte copy
  const int4* vsrc = reinterpret_cast<const int4*>(src_row + (int64_t)(hq + hkv) * D);
  int4* vd = reinterpret_cast<int4*>(pool + vdst);
  for (int i = threadIdx.x; i < vv; i += blockDim.x) vd[i] = vsrc[i];
}

template <typename T>
__global__ void __launch_bounds__(256) silu_mul_kernel(const T* __restrict__ gu,
                                                       T* __restrict__ out, int n, int F) {
  pdl_wait();
  constexpr int V = 16 / sizeof(T);
  const int64_t per_row = F / V;
  const int64_t total = (int64_t)n * per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / per_row, c = (i % per_row) * V;
    float g[V], u[V], r[V];
    load_vec<T, V>(gu + row * 2 * F + c, g);
    load_vec<T, V>(gu + row * 2 * F + F + c, u);
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const float sg = to_f(from_f<T>(g[k] / (1.f + expf(-g[k]))));  // act rounded like the reference
      r[k] = sg * u[k];
    }
    store_vec<T, V>(out + row * F + c, r);
  }
}

}  // namespace be

using namespace be;

extern "C" int be_add_rmsnorm(void* residual, const void* delta, const void* weight, void* out,
                              int rows, int hidden, float eps, int dtype, void* stream) {
  const int V = 16 / dtype_size(dtype);
  if (rows < 0 || hidden % V || hidden > 256 * 8 * V) {
    set_error("be_add_rmsnorm: hidden %d must be a multiple of %d and <= %d", hidden, V, 256 * 8 * V);
    return BE_EINVAL;
  }
  if (rows == 0) return BE_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const int threads = 256;
  switch (dtype) {
    case BE_BF16:
      BE_CUDA_CHECK(launch_pdl(add_rmsnorm_kernel<__nv_bfloat16>, rows, threads, 0, st,
                               (__nv_bfloat16*)residual, (const __nv_bfloat16*)delta,
                               (const __nv_bfloat16*)weight, (__nv_bfloat16*)out, hidden, eps));
      break;
    case BE_F16:
      BE_CUDA_CHECK(launch_pdl(add_rmsnorm_kernel<__half>, rows, threads, 0, st, (__half*)residual,
                               (const __half*)delta, (const __half*)weight, (__half*)out, hidden,
                               eps));
      break;
    default:
      BE_CUDA_CHECK(launch_pdl(add_rmsnorm_kernel<float>, rows, threads, 0, st, (float*)residual,
                               (const float*)delta, (const float*)weight, (float*)out, hidden, eps));
  }
  BE_LAUNCH_CHECK();
  return BE_OK;
}

extern "C" int be_rope_qkv_append(void* qkv, int64_t row_stride, int n, int num_qo_heads,
                                  int num_kv_heads, int head_dim, const int32_t* positions,
                                  const float* inv_freq, void* paged_kv_cache, int num_pages,
                                  int page_size, const int32_t* write_page,
                                  const int32_t* write_pos, int rope_k_in_place, int dtype,
                                  void* stream) {
  if (n < 0 || head_dim % 2 || num_kv_heads < 1) {
    set_error("be_rope_qkv_append: invalid shape");
    return BE_EINVAL;
  }
  if (n == 0) return BE_OK;
  const int64_t warps = (int64_t)n * (num_qo_heads + 2 * num_kv_heads);
  const int threads = 256;
  const int blocks = (int)((warps * 32 + threads - 1) / threads);
  cudaStream_t st = (cudaStream_t)stream;
  const int V = 16 / dtype_size(dtype);
  const bool rows_form = (head_dim / 2) % V == 0 && head_dim / 2 <= 256 && row_stride % V == 0 &&
                         ((uintptr_t)qkv & 15) == 0 && ((uintptr_t)paged_kv_cache & 15) == 0;
  if (rows_form) {
#define BE_ROPE_ROWS(T)                                                                        \
  BE_CUDA_CHECK(launch_pdl(rope_append_rows_kernel<T>, n, threads, 0, st, (T*)qkv, row_stride, n, \
                           num_qo_heads, num_kv_heads, head_dim, positions, inv_freq,            \
                           (T*)paged_kv_cache, num_pages, page_size, write_page, write_pos,      \
                           rope_k_in_place))
    switch (dtype) {
      case BE_BF16: BE_ROPE_ROWS(__nv_bfloat16); break;
      case BE_F16: BE_ROPE_ROWS(__half); break;
      default: BE_ROPE_ROWS(float);
    }
#undef BE_ROPE_ROWS
    BE_LAUNCH_CHECK();
    return BE_OK;
  }
#define BE_ROPE(T)                                                                           \
  BE_CUDA_CHECK(launch_pdl(rope_append_kernel<T>, blocks, threads, 0, st, (T*)qkv, row_stride, n, \
                           num_qo_heads, num_kv_heads, head_dim, positions, inv_freq,            \
                           (T*)paged_kv_cache, num_pages, page_size, write_page, write_pos,      \
                           rope_k_in_place))
  switch (dtype) {
    case BE_BF16: BE_ROPE(__nv_bfloat16); break;
    case BE_F16: BE_ROPE(__half); break;
    default: BE_ROPE(float);
  }
#undef BE_ROPE
  BE_LAUNCH_CHECK();
  return BE_OK;
}

extern "C" int be_silu_mul(const void* gate_up, void* out, int n, int ffn, int dtype,
                           void* stream) {
  const int V = 16 / dtype_size(dtype);
  if (n < 0 || ffn % V) {
    set_error("be_silu_mul: ffn %d must be a multiple of %d", ffn, V);
    return BE_EINVAL;
  }
  if (n == 0) return BE_OK;
  const int64_t total = (int64_t)n * (ffn / V);
  const int threads = 256;
  const int blocks = (int)std::min<int64_t>((total + threads - 1) / threads, 148 * 16);
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case BE_BF16:
      BE_CUDA_CHECK(launch_pdl(silu_mul_kernel<__nv_bfloat16>, blocks, threads, 0, st,
                               (const __nv_bfloat16*)gate_up, (__nv_bfloat16*)out, n, ffn));
      break;
    case BE_F16:
      BE_CUDA_CHECK(launch_pdl(silu_mul_kernel<__half>, blocks, threads, 0, st,
                               (const __half*)gate_up, (__half*)out, n, ffn));
      break;
    default:
      BE_CUDA_CHECK(launch_pdl(silu_mul_kernel<float>, blocks, threads, 0, st,
                               (const float*)gate_up, (float*)out, n, ffn));
  }
  BE_LAUNCH_CHECK();
  return BE_OK;
}
