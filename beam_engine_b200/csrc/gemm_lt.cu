// Decode projections through cuBLASLt with a per-shape algorithm choice.
//
// The step's GEMMs (q/k/v, o, gate/up, down, lm_head at 128 rows) are plain
// library GEMMs; torch.mm takes cuBLASLt's first heuristic for each.  Here the
// first call of a shape (outside stream capture) times the heuristic's top
// candidates -- split-K variants included -- on the caller's stream and keeps
// the fastest; later calls, and calls inside a capture, reuse it.
//
//   Y[T][N] = X[T][K] * W[N][K]^T    (row-major, bf16 operands, fp32 accumulate)
// is computed column-major as Y^T (N x T) = op_T(W_cm: K x N) * X_cm (K x T).
#include <cublasLt.h>

namespace be {

struct LtKey {
  int T, N, K, out;
  int64_t ldx, ldw, ldy;
  bool operator==(const LtKey& o) const {
    return T == o.T && N == o.N && K == o.K && out == o.out && ldx == o.ldx && ldw == o.ldw &&
           ldy == o.ldy;
  }
};
struct LtKeyHash {
  size_t operator()(const LtKey& k) const {
    return ((size_t)k.T * 1315423911u) ^ ((size_t)k.N * 2654435761u) ^ ((size_t)k.K * 97u) ^
           ((size_t)k.out << 7) ^ (size_t)(k.ldx * 131 + k.ldw * 17 + k.ldy);
  }
};
struct LtPlan {
  cublasLtMatmulDesc_t op = nullptr;
  cublasLtMatrixLayout_t a = nullptr, b = nullptr, c = nullptr;
  cublasLtMatmulAlgo_t algo;
  size_t ws_needed = 0;
  bool tuned = false;
};

static cublasLtHandle_t lt_handle() {
  static std::mutex mu;
  static cublasLtHandle_t h[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  if (dev >= 0 && dev < 64 && !h[dev]) cublasLtCreate(&h[dev]);
  return dev >= 0 && dev < 64 ? h[dev] : nullptr;
}

#define BE_LT_CHECK(expr)                                                     \
  do {                                                                        \
    cublasStatus_t _s = (expr);                                               \
    if (_s != CUBLAS_STATUS_SUCCESS) {                                        \
      ::be::set_error("%s: cublas status %d (%s:%d)", #expr, (int)_s, __FILE__, \
                      __LINE__);                                              \
      return BE_ECUDA;                                                        \
    }                                                                         \
  } while (0)

static int lt_make(const LtKey& k, LtPlan* p) {
  const cudaDataType_t out_t = k.out == BE_BF16 ? CUDA_R_16BF : CUDA_R_32F;
  BE_LT_CHECK(cublasLtMatmulDescCreate(&p->op, CUBLAS_COMPUTE_32F, CUDA_R_32F));
  const cublasOperation_t ta = CUBLAS_OP_T, tb = CUBLAS_OP_N;
  BE_LT_CHECK(cublasLtMatmulDescSetAttribute(p->op, CUBLASLT_MATMUL_DESC_TRANSA, &ta, sizeof(ta)));
  BE_LT_CHECK(cublasLtMatmulDescSetAttribute(p->op, CUBLASLT_MATMUL_DESC_TRANSB, &tb, sizeof(tb)));
  BE_LT_CHECK(cublasLtMatrixLayoutCreate(&p->a, CUDA_R_16BF, k.K, k.N, k.ldw));
  BE_LT_CHECK(cublasLtMatrixLayoutCreate(&p->b, CUDA_R_16BF, k.K, k.T, k.ldx));
  BE_LT_CHECK(cublasLtMatrixLayoutCreate(&p->c, out_t, k.N, k.T, k.ldy));
  return BE_OK;
}

}  // namespace be

using namespace be;

extern "C" int be_gemm_lt(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y,
                          int64_t ldy, int T, int N, int K, int out_dtype, void* workspace,
                          int64_t workspace_bytes, void* stream) {
  if (!x || !w || !y || T < 1 || N < 1 || K < 1 || ldx < K || ldw < K || ldy < N ||
      (out_dtype != BE_BF16 && out_dtype != BE_F32)) {
    set_error("be_gemm_lt: invalid arguments");
    return BE_EINVAL;
  }
  static std::mutex mu;
  static std::unordered_map<LtKey, LtPlan, LtKeyHash> cache;
  cublasLtHandle_t h = lt_handle();
  if (!h) {
    set_error("be_gemm_lt: cublasLtCreate failed");
    return BE_ECUDA;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const LtKey key{T, N, K, out_dtype, ldx, ldw, ldy};
  const float alpha = 1.f, beta = 0.f;
  std::lock_guard<std::mutex> lk(mu);
  LtPlan& p = cache[key];
  if (!p.op) {
    int rc = lt_make(key, &p);
    if (rc != BE_OK) return rc;
  }
  if (!p.tuned) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    BE_CUDA_CHECK(cudaStreamIsCapturing(st, &cs));
    cublasLtMatmulPreference_t pref;
    BE_LT_CHECK(cublasLtMatmulPreferenceCreate(&pref));
    uint64_t wsb = (uint64_t)std::max<int64_t>(workspace_bytes, 0);
    BE_LT_CHECK(cublasLtMatmulPreferenceSetAttribute(
        pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &wsb, sizeof(wsb)));
    cublasLtMatmulHeuristicResult_t res[16];
    int n_res = 0;
    cublasStatus_t hs = cublasLtMatmulAlgoGetHeuristic(h, p.op, p.a, p.b, p.c, p.c, pref, 16, res,
                                                       &n_res);
    cublasLtMatmulPreferenceDestroy(pref);
    if (hs != CUBLAS_STATUS_SUCCESS || n_res == 0) {
      set_error("be_gemm_lt: no cuBLASLt algorithm for T %d N %d K %d", T, N, K);
      return BE_ECUDA;
    }
    int best = 0;
    if (cs == cudaStreamCaptureStatusNone && n_res > 1) {   // time the candidates once
      cudaEvent_t e0, e1;
      BE_CUDA_CHECK(cudaEventCreate(&e0));
      BE_CUDA_CHECK(cudaEventCreate(&e1));
      float best_ms = 1e30f;
      for (int i = 0; i < n_res; ++i) {
        if (res[i].workspaceSize > wsb) continue;
        bool ok = true;
        for (int r = 0; r < 2 && ok; ++r)   // warm-up
          ok = cublasLtMatmul(h, p.op, &alpha, w, p.a, x, p.b, &beta, y, p.c, y, p.c, &res[i].algo,
                              workspace, wsb, st) == CUBLAS_STATUS_SUCCESS;
        if (!ok) continue;
        BE_CUDA_CHECK(cudaEventRecord(e0, st));
        for (int r = 0; r < 5; ++r)
          cublasLtMatmul(h, p.op, &alpha, w, p.a, x, p.b, &beta, y, p.c, y, p.c, &res[i].algo,
                         workspace, wsb, st);
        BE_CUDA_CHECK(cudaEventRecord(e1, st));
        BE_CUDA_CHECK(cudaEventSynchronize(e1));
        float ms = 0.f;
        BE_CUDA_CHECK(cudaEventElapsedTime(&ms, e0, e1));
        if (ms < best_ms) {
          best_ms = ms;
          best = i;
        }
      }
      cudaEventDestroy(e0);
      cudaEventDestroy(e1);
    }
    if (cs == cudaStreamCaptureStatusNone) p.tuned = true;
    p.algo = res[best].algo;
    p.ws_needed = res[best].workspaceSize;
  }
  if (p.ws_needed > (size_t)std::max<int64_t>(workspace_bytes, 0)) {
    set_error("be_gemm_lt: algorithm needs %zu bytes of workspace", p.ws_needed);
    return BE_ECAPACITY;
  }
  BE_LT_CHECK(cublasLtMatmul(h, p.op, &alpha, w, p.a, x, p.b, &beta, y, p.c, y, p.c, &p.algo,
                             workspace, (size_t)workspace_bytes, st));
  return BE_OK;
}
