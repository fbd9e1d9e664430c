// Beam scoring on the device: logits -> log_softmax -> top-k in one launch.
//
// The reference scores every beam as `logits / temperature -> log_softmax ->
// topk(2W)` (beam.py:266-317) with three library ops; torch's top-k alone is
// ~10 launches per call on a [128, 128256] block.  Here one CTA owns one row:
//   * pass 1 streams the row from HBM with 16-byte loads: each lane's maximum;
//     from the 1024 lane maxima the row max and tau, the k-th largest lane
//     maximum -- a lower bound of the row's k-th largest value;
//   * pass 2 reads the row again (from L2): the sum of exponentials against the
//     exact max, and every warp keeps the top KMAX (value, id) pairs of its
//     chunk as a list sorted by (value desc, id asc), KMAX / 32 entries per
//     lane, offered only the values that reach tau (a handful per warp,
//     instead of a few hundred insertions while a list fills up);
//   * the warps' lists meet in shared memory, where every entry finds its rank
//     among all lists by binary search (no serial merge);
//   * out: log-probabilities (x - max) - log(sum) of the k best with global
//     vocabulary ids, or -- for a vocabulary slice under tensor parallelism --
//     the raw scaled logits plus the slice's max and sum for a cross-rank
//     log-sum-exp.
// HBM-bound: rows x vocab x 4 bytes read once.
#include "common.cuh"

namespace be {

constexpr int TK_THREADS = 1024;
constexpr int TK_WARPS = TK_THREADS / 32;
constexpr int TK_KMAX = 64;            // entries per list (k <= 64)
constexpr int TK_PER_LANE = TK_KMAX / 32;

// (value, id) order: larger value first, equal values by smaller id
__device__ __forceinline__ bool tk_better(float a, int ia, float b, int ib) {
  return a > b || (a == b && ia < ib);
}

// Warp-wide sorted list: entry e = slot * 32 + lane (slot 0 holds entries 0-31).
struct WarpTopK {
  float v[TK_PER_LANE];
  int id[TK_PER_LANE];

  __device__ __forceinline__ void init() {
#pragma unroll
    for (int s = 0; s < TK_PER_LANE; ++s) {
      v[s] = -INFINITY;
      id[s] = INT_MAX;
    }
  }
  // value / id of entry k - 1 (the admission threshold), on every lane
  __device__ __forceinline__ void kth(int k, float& tv, int& ti) const {
    const int e = k - 1, s = e >> 5, l = e & 31;
    float vv = v[0];
    int ii = id[0];
#pragma unroll
    for (int q = 1; q < TK_PER_LANE; ++q)
      if (s == q) {
        vv = v[q];
        ii = id[q];
      }
    tv = __shfl_sync(0xffffffffu, vv, l);
    ti = __shfl_sync(0xffffffffu, ii, l);
  }
  // insert (x, ix) -- warp-uniform arguments -- keeping the list sorted
  __device__ __forceinline__ void insert(float x, int ix) {
    const int lane = threadIdx.x & 31;
    // position = number of entries better than the candidate
    int pos = 0;
#pragma unroll
    for (int s = 0; s < TK_PER_LANE; ++s)
      pos += __popc(__ballot_sync(0xffffffffu, tk_better(v[s], id[s], x, ix)));
    // shift entries >= pos down by one (entry e takes entry e - 1)
    float carry_v = -INFINITY;
    int carry_i = INT_MAX;
#pragma unroll
    for (int s = 0; s < TK_PER_LANE; ++s) {
      float up_v = __shfl_up_sync(0xffffffffu, v[s], 1);
      int up_i = __shfl_up_sync(0xffffffffu, id[s], 1);
      const float last_v = __shfl_sync(0xffffffffu, v[s], 31);
      const int last_i = __shfl_sync(0xffffffffu, id[s], 31);
      if (lane == 0) {
        up_v = carry_v;
        up_i = carry_i;
      }
      const int e = s * 32 + lane;
      if (e > pos) {
        v[s] = up_v;
        id[s] = up_i;
      } else if (e == pos) {
        v[s] = x;
        id[s] = ix;
      }
      carry_v = last_v;
      carry_i = last_i;
    }
  }
  // offer one candidate per lane; those that beat entry k - 1 go in, lowest lane first
  __device__ __forceinline__ void offer(float x, int ix, int k, float& tv, int& ti) {
    unsigned m = __ballot_sync(0xffffffffu, tk_better(x, ix, tv, ti));
    while (m) {
      const int src = __ffs(m) - 1;
      const float cx = __shfl_sync(0xffffffffu, x, src);
      const int ci = __shfl_sync(0xffffffffu, ix, src);
      insert(cx, ci);
      kth(k, tv, ti);
      m &= ~(1u << src);
      m &= __ballot_sync(0xffffffffu, tk_better(x, ix, tv, ti));
    }
  }
};

__global__ void __launch_bounds__(TK_THREADS) logsoftmax_topk_kernel(
    const float* __restrict__ logits, int64_t ld, int v, float temperature, int k,
    int64_t vocab_offset, int full_vocab, float* __restrict__ out_val, int64_t* __restrict__ out_idx,
    float* __restrict__ row_max, float* __restrict__ row_sum) {
  __shared__ float s_v[TK_WARPS][TK_KMAX];
  __shared__ int s_i[TK_WARPS][TK_KMAX];
  __shared__ float s_s[TK_WARPS];
  pdl_wait();
  const int row = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float* x = logits + (int64_t)row * ld;
  const bool scale = temperature != 1.0f;
  // contiguous chunk per warp (multiple of 128 elements so float4 loads stay aligned)
  const int per_warp = ((v + TK_WARPS - 1) / TK_WARPS + 127) / 128 * 128;
  const int c0 = min(v, warp * per_warp), c1 = min(v, c0 + per_warp);
  const bool vec = ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  __shared__ float s_lmax[TK_THREADS];
  __shared__ float s_tau;
  auto load4 = [&](int col) {   // 4 scaled values from col (-inf past the chunk's end)
    float4 r;
    if (vec && col + 3 < c1) {
      r = __ldcg(reinterpret_cast<const float4*>(x + col));   // kept in L2 for the second pass
    } else {
      r.x = col < c1 ? x[col] : -INFINITY;
      r.y = col + 1 < c1 ? x[col + 1] : -INFINITY;
      r.z = col + 2 < c1 ? x[col + 2] : -INFINITY;
      r.w = col + 3 < c1 ? x[col + 3] : -INFINITY;
    }
    if (scale) {
      r.x = r.x / temperature;
      r.y = r.y / temperature;
      r.z = r.z / temperature;
      r.w = r.w / temperature;
    }
    return r;
  };
  // Pass 1 (from HBM): each lane's maximum.  TK_DEPTH 16-byte loads per lane in
  // flight before any is used.
  constexpr int TK_DEPTH = 4;
  float lmax = -INFINITY;
  for (int base0 = c0; base0 < c1; base0 += 128 * TK_DEPTH) {
    float4 buf[TK_DEPTH];
#pragma unroll
    for (int u = 0; u < TK_DEPTH; ++u) buf[u] = load4(base0 + u * 128 + lane * 4);
#pragma unroll
    for (int u = 0; u < TK_DEPTH; ++u)
      lmax = fmaxf(lmax, fmaxf(fmaxf(buf[u].x, buf[u].y), fmaxf(buf[u].z, buf[u].w)));
  }
  // The row max, and tau = the k-th largest of the 1024 lane maxima: they are
  // k distinct elements of the row at least as large as tau, so tau is a lower
  // bound of the row's k-th largest value and nothing below it can be selected.
  s_lmax[tid] = lmax;
  __syncthreads();
  {
    int above = 0, tie_before = 0;
    for (int j = 0; j < TK_THREADS; ++j) {      // every thread reads the same word: broadcast
      const float o = s_lmax[j];
      above += o > lmax;
      tie_before += (o == lmax) & (j < tid);
    }
    if (above + tie_before == k - 1) s_tau = lmax;
  }
  float m = -INFINITY;
  for (int j = lane; j < TK_THREADS; j += 32) m = fmaxf(m, s_lmax[j]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __syncthreads();
  const float tau = s_tau;
  // Pass 2 (from L2): the sum of exponentials against the exact max, and the
  // warp's top-k list offered only what reaches tau (a handful per warp).
  WarpTopK tk;
  tk.init();
  float tv = -INFINITY;
  int ti = INT_MAX;
  float s = 0.f;
  const float m0 = m == -INFINITY ? 0.f : m;   // a row of -inf sums to 0, not NaN
  for (int base0 = c0; base0 < c1; base0 += 128 * TK_DEPTH) {
    float4 buf[TK_DEPTH];
#pragma unroll
    for (int u = 0; u < TK_DEPTH; ++u) buf[u] = load4(base0 + u * 128 + lane * 4);
#pragma unroll
    for (int u = 0; u < TK_DEPTH; ++u) {
      if (base0 + u * 128 >= c1) break;              // warp-uniform
      const int col = base0 + u * 128 + lane * 4;
      const float e[4] = {buf[u].x, buf[u].y, buf[u].z, buf[u].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) s += __expf(e[i] - m0);   // -inf past the end adds 0
      const float bm = fmaxf(fmaxf(e[0], e[1]), fmaxf(e[2], e[3]));
      if (__any_sync(0xffffffffu, bm >= tau)) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const bool in = col + i < c1 && e[i] >= tau;
          tk.offer(in ? e[i] : -INFINITY, in ? col + i : INT_MAX, k, tv, ti);
        }
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
#pragma unroll
  for (int q = 0; q < TK_PER_LANE; ++q) {
    s_v[warp][q * 32 + lane] = tk.v[q];
    s_i[warp][q * 32 + lane] = tk.id[q];
  }
  if (lane == 0) s_s[warp] = s;
  __syncthreads();
  s = s_s[lane];   // every warp sums the 32 warp partials (same order: same bits)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float log_s = logf(s);
  // the block's top k: the first k entries of every warp's sorted list are
  // ranked against all other lists at once (rank = entries strictly better,
  // a binary search per list); (value, id) pairs are distinct, so ranks
  // 0..k-1 are each taken by exactly one entry
  for (int i = tid; i < TK_WARPS * k; i += TK_THREADS) {
    const int w = i / k, e = i - w * k;
    const float xv = s_v[w][e];
    const int xi = s_i[w][e];
    int rank = e;
    for (int w2 = 0; w2 < TK_WARPS; ++w2) {
      if (w2 == w) continue;
      int lo = 0, hi = k;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (tk_better(s_v[w2][mid], s_i[w2][mid], xv, xi)) lo = mid + 1;
        else hi = mid;
      }
      rank += lo;
      if (rank >= k) break;
    }
    if (rank < k) {
      out_val[(int64_t)row * k + rank] = full_vocab ? (xv - m) - log_s : xv;
      out_idx[(int64_t)row * k + rank] = (int64_t)xi + vocab_offset;
    }
  }
  if (!full_vocab && tid == 0) {
    row_max[row] = m;
    row_sum[row] = s;
  }
}

}  // namespace be

using namespace be;

extern "C" int be_logsoftmax_topk(const float* logits, int64_t ld, int rows, int v, float temperature,
                                  int k, int64_t vocab_offset, int full_vocab, float* out_val,
                                  int64_t* out_idx, float* row_max, float* row_sumexp, void* stream) {
  if (!logits || !out_val || !out_idx || rows < 0 || v < 1 || k < 1 || k > TK_KMAX || k > v ||
      ld < v || !(temperature > 0.f)) {
    set_error("be_logsoftmax_topk: invalid arguments (rows %d, v %d, k %d <= %d, ld %lld)", rows, v,
              k, TK_KMAX, (long long)ld);
    return BE_EINVAL;
  }
  if (!full_vocab && (!row_max || !row_sumexp)) {
    set_error("be_logsoftmax_topk: a vocabulary slice needs row_max and row_sumexp");
    return BE_EINVAL;
  }
  if (rows == 0) return BE_OK;
  BE_CUDA_CHECK(launch_pdl(logsoftmax_topk_kernel, rows, TK_THREADS, 0, (cudaStream_t)stream,
                           logits, ld, v, temperature, k, vocab_offset, full_vocab, out_val, out_idx,
                           row_max, row_sumexp));
  BE_LAUNCH_CHECK();
  return BE_OK;
}

// ---------------------------------------------------------------------------
// Global top-W of every prompt on the device: VanillaBeamSearchStrategy
// .select_candidates (src/beam_engine/beam_strategy.py:433-488).  Candidate c
// of prompt s (c in seg_ptr[s]..seg_ptr[s+1]) offers its top-k children with
// accumulated score parent_scores[c] + logps[c][j] (double, as the reference's
// Python floats); the prompt keeps the beam_size best by a stable descending
// sort of the flattened (candidate, j) list: equal scores keep the earlier
// candidate, then the earlier top-k position.  One CTA per prompt: every
// entry counts the entries ranked before it.  Entries at top-k position
// j >= beam_size cannot be selected (the row is sorted, so j entries of the
// same candidate rank before it) and only take part as competitors.
// ---------------------------------------------------------------------------
namespace be {

constexpr int SEL_THREADS = 512;
constexpr int SEL_MAX = 8192;          // entries per prompt (candidates x k) held in shared memory

__global__ void __launch_bounds__(SEL_THREADS) vanilla_select_kernel(
    const int32_t* __restrict__ seg_ptr, int k, const double* __restrict__ parent_scores,
    const float* __restrict__ logps, const int64_t* __restrict__ tokens, int beam_size,
    int cap_entries, int32_t* __restrict__ sel_parent, int32_t* __restrict__ sel_token,
    double* __restrict__ sel_score) {
  extern __shared__ double s_tot[];
  pdl_wait();
  const int s = blockIdx.x;
  const int c0 = seg_ptr[s], c1 = seg_ptr[s + 1];
  const int m = (c1 - c0) * k;
  if (m > cap_entries || c1 < c0) {                // more than the launch's shared memory
    if (threadIdx.x == 0) flag_range_error();
    return;
  }
  for (int e = threadIdx.x; e < m; e += blockDim.x) {
    const int c = c0 + e / k;
    s_tot[e] = parent_scores[c] + (double)logps[(int64_t)c * k + e % k];
  }
  __syncthreads();
  const int jmax = min(k, beam_size);
  const int cands = (c1 - c0) * jmax;
  for (int x = threadIdx.x; x < cands; x += blockDim.x) {
    const int e = (x / jmax) * k + x % jmax;
    const double te = s_tot[e];
    int rank = 0;
    for (int f = 0; f < m && rank < beam_size; ++f) {
      const double tf = s_tot[f];
      rank += (tf > te) || (tf == te && f < e);
    }
    if (rank < beam_size) {
      const int c = c0 + e / k;
      const int64_t o = (int64_t)s * beam_size + rank;
      sel_parent[o] = c;
      sel_token[o] = (int32_t)tokens[(int64_t)c * k + e % k];
      sel_score[o] = te;
    }
  }
  for (int r = min(beam_size, m) + threadIdx.x; r < beam_size; r += blockDim.x)
    sel_parent[(int64_t)s * beam_size + r] = -1;
}

}  // namespace be

extern "C" int be_vanilla_select_device(int nseg, const int32_t* seg_ptr, int k,
                                        const double* parent_scores, const float* logps,
                                        const int64_t* tokens, int beam_size, int max_seg_cands,
                                        int32_t* sel_parent, int32_t* sel_token,
                                        double* sel_score, void* stream) {
  using namespace be;
  if (nseg < 0 || k < 1 || beam_size < 1 || max_seg_cands < 0 || !seg_ptr || !parent_scores ||
      !logps || !tokens || !sel_parent || !sel_token || !sel_score) {
    set_error("be_vanilla_select_device: invalid arguments");
    return BE_EINVAL;
  }
  if ((int64_t)max_seg_cands * k > SEL_MAX) {
    set_error("be_vanilla_select_device: %d candidates x top-%d exceed %d entries per prompt",
              max_seg_cands, k, SEL_MAX);
    return BE_EINVAL;
  }
  if (nseg == 0) return BE_OK;
  const size_t smem = (size_t)max_seg_cands * k * sizeof(double);
  static bool set = false;
  if (!set) {
    BE_CUDA_CHECK(cudaFuncSetAttribute(vanilla_select_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)(SEL_MAX * sizeof(double))));
    set = true;
  }
  BE_CUDA_CHECK(launch_pdl(vanilla_select_kernel, nseg, SEL_THREADS, smem, (cudaStream_t)stream,
                           seg_ptr, k, parent_scores, logps, tokens, beam_size,
                           max_seg_cands * k, sel_parent, sel_token, sel_score));
  return BE_OK;
}

// ---------------------------------------------------------------------------
// Diverse beam search selection on the device, hamming penalty:
// DiverseBeamSearchStrategy.select_candidates (src/beam_engine/beam_strategy.py:
// 173-317, penalty :105-125), the same outputs as the host be_diverse_select.
// One CTA per prompt.  The prompt's (candidate, j) choices are first ordered by
// log-probability (stable, descending): ord[e] is that position.  Group g
// scores every choice not yet taken as (logp - pen) / (len + 1) ** lpen, with
// pen = diversity_penalty when an earlier group of this step took the same
// token, and takes the bpg = max(1, beam_size / num_groups) best by (score
// descending, ord ascending) -- the host's second stable sort -- each choice
// counting the untaken choices ranked before it.  Picks are listed per parent
// (parents ascending, picks in pick order) and the first beam_size kept, which
// is what dropping children from the end, last parent first, leaves.
// ---------------------------------------------------------------------------
namespace be {

constexpr int DIV_PICKS = 1024;        // picks per prompt (num_groups * bpg) held in shared memory

__global__ void __launch_bounds__(SEL_THREADS) diverse_select_kernel(
    const int32_t* __restrict__ seg_ptr, int k, const double* __restrict__ parent_scores,
    const int32_t* __restrict__ tokens, const double* __restrict__ logps,
    const int32_t* __restrict__ seq_ptr, int beam_size, int num_groups, double dpen, double lpen,
    int cap_entries, int32_t* __restrict__ child_ptr, int32_t* __restrict__ child_tokens,
    double* __restrict__ child_scores, int32_t* __restrict__ new_seg_ptr) {
  extern __shared__ __align__(16) unsigned char div_smem[];
  __shared__ int picks[DIV_PICKS];
  __shared__ int pick_tok[DIV_PICKS];
  pdl_wait();
  const int s = blockIdx.x;
  const int c0 = seg_ptr[s], c1 = seg_ptr[s + 1];
  const int m = (c1 - c0) * k;
  if (c1 < c0 || m > cap_entries) {
    if (threadIdx.x == 0) flag_range_error();
    return;
  }
  const int bpg = max(1, beam_size / num_groups);
  const int npick_all = min(num_groups * bpg, m);   // sum over groups of min(bpg, untaken)
  const int kept = min(beam_size, npick_all);
  int off = 0;                                      // kept children of the earlier prompts
  for (int t = 0; t < s; ++t)
    off += min(beam_size, min(num_groups * bpg, (seg_ptr[t + 1] - seg_ptr[t]) * k));
  double* score = reinterpret_cast<double*>(div_smem);
  int* ord = reinterpret_cast<int*>(score + cap_entries);
  unsigned char* taken = reinterpret_cast<unsigned char*>(ord + cap_entries);
  const double* lp = logps + (int64_t)c0 * k;
  const int32_t* tk = tokens + (int64_t)c0 * k;
  for (int e = threadIdx.x; e < m; e += blockDim.x) {
    const double le = lp[e];
    int r = 0;
    for (int f = 0; f < m; ++f) {
      const double lf = lp[f];
      r += (lf > le) || (lf == le && f < e);
    }
    ord[e] = r;
    taken[e] = 0;
  }
  int npick = 0;
  for (int g = 0; g < num_groups && npick < npick_all; ++g) {
    __syncthreads();
    for (int e = threadIdx.x; e < m; e += blockDim.x) {
      if (taken[e]) continue;
      const int32_t tok = tk[e];
      double pen = 0.0;
      for (int q = 0; q < npick; ++q)
        if (pick_tok[q] == tok) {
          pen = dpen;
          break;
        }
      double sc = lp[e] - pen;
      if (lpen != 0.0) {
        const int c = c0 + e / k;
        const double len1 = (double)(seq_ptr[c + 1] - seq_ptr[c]) + 1.0;
        sc = sc / (lpen == 1.0 ? len1 : pow(len1, lpen));
      }
      score[e] = sc;
    }
    __syncthreads();
    const int take = min(bpg, m - npick);
    for (int e = threadIdx.x; e < m; e += blockDim.x) {
      if (taken[e]) continue;
      const double se = score[e];
      const int oe = ord[e];
      int r = 0;
      for (int f = 0; f < m && r < take; ++f) {
        if (taken[f]) continue;
        const double sf = score[f];
        r += (sf > se) || (sf == se && ord[f] < oe);
      }
      if (r < take) picks[npick + r] = e;
    }
    __syncthreads();
    for (int r = threadIdx.x; r < take; r += blockDim.x) {
      const int e = picks[npick + r];
      taken[e] = 1;
      pick_tok[npick + r] = tk[e];
    }
    npick += take;
  }
  __syncthreads();
  // parent-major order of the picks; the first `kept` are the children
  for (int r = threadIdx.x; r < npick; r += blockDim.x) {
    const int e = picks[r];
    const int pe = e / k;
    int pos = 0;
    for (int q = 0; q < npick; ++q) {
      const int pq = picks[q] / k;
      pos += (pq < pe) || (pq == pe && q < r);
    }
    if (pos < kept) {
      child_tokens[off + pos] = tk[e];
      child_scores[off + pos] = parent_scores[c0 + pe] + lp[e];
    }
  }
  for (int i = threadIdx.x; i < c1 - c0; i += blockDim.x) {
    int cnt = 0;
    for (int q = 0; q < npick; ++q) cnt += picks[q] / k <= i;
    child_ptr[c0 + i + 1] = off + min(kept, cnt);
  }
  if (threadIdx.x == 0) {
    new_seg_ptr[s + 1] = off + kept;
    if (s == 0) {
      child_ptr[0] = 0;
      new_seg_ptr[0] = 0;
    }
  }
}

}  // namespace be

extern "C" int be_diverse_select_device(int nseg, const int32_t* seg_ptr, int k,
                                        const double* parent_scores, const int32_t* tokens,
                                        const double* logps, const int32_t* seq_ptr,
                                        int beam_size, int num_groups, double diversity_penalty,
                                        int diversity_type, double length_penalty,
                                        int max_seg_cands, int32_t* child_ptr,
                                        int32_t* child_tokens, double* child_scores,
                                        int32_t* new_seg_ptr, void* stream) {
  using namespace be;
  if (nseg < 0 || k < 1 || beam_size < 1 || num_groups < 1 || max_seg_cands < 0 || !seg_ptr ||
      !parent_scores || !tokens || !logps || !seq_ptr || !child_ptr || !child_tokens ||
      !child_scores || !new_seg_ptr) {
    set_error("be_diverse_select_device: invalid arguments");
    return BE_EINVAL;
  }
  if (diversity_type != 0) {
    set_error("be_diverse_select_device: only the hamming penalty runs on the device "
              "(be_diverse_select serves the cumulative one)");
    return BE_ENOTSUP;
  }
  if ((int64_t)max_seg_cands * k > SEL_MAX) {
    set_error("be_diverse_select_device: %d candidates x top-%d exceed %d entries per prompt",
              max_seg_cands, k, SEL_MAX);
    return BE_EINVAL;
  }
  const int bpg = std::max(1, beam_size / num_groups);
  if ((int64_t)num_groups * bpg > DIV_PICKS) {
    set_error("be_diverse_select_device: %d groups x %d picks exceed %d per prompt", num_groups,
              bpg, DIV_PICKS);
    return BE_EINVAL;
  }
  if (nseg == 0) return BE_OK;
  const int cap = std::max(1, max_seg_cands * k);
  const size_t smem = (size_t)cap * (sizeof(double) + sizeof(int) + 1);
  static bool set = false;
  if (!set) {
    BE_CUDA_CHECK(cudaFuncSetAttribute(diverse_select_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)(SEL_MAX * (sizeof(double) + sizeof(int) + 1))));
    set = true;
  }
  BE_CUDA_CHECK(launch_pdl(diverse_select_kernel, nseg, SEL_THREADS, smem, (cudaStream_t)stream,
                           seg_ptr, k, parent_scores, tokens, logps, seq_ptr, beam_size,
                           num_groups, diversity_penalty, length_penalty, cap, child_ptr,
                           child_tokens, child_scores, new_seg_ptr));
  return BE_OK;
}
