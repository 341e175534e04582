// CUDA-core GEMM kernels and the mtp_gemm dispatcher.
//   gemm_simt  64x64 tiles, 4x4 outputs per thread: the fp32 model path (exact fp32
//              products, used for parity with the fp32 reference) and odd shapes.
//   gemv       small-M (decode) kernel: one warp per pair of weight rows streams the rows
//              with 16-byte loads and dots them with up to 8 token vectors at a time.
#include "common.cuh"

namespace mtp {

bool gemm_tc_eligible(const void *A, const void *B, int M, int N, int K, int lda, int ldb);
int gemm_tc(const void *A, const void *B, void *C, int M, int N, int K, int lda, int ldb, int ldc, int c_dtype,
            int epi, const void *bias, int bias_dtype, cudaStream_t stream);

struct EpiArgs {
  void *C;
  int ldc, c_dtype, epi;
  const void *bias;
  int bias_dtype;
};

__device__ __forceinline__ void epi_store(const EpiArgs &e, int m, int n, float v) {
  if (e.epi != MTP_EPI_STORE) {
    const float b = e.bias_dtype == MTP_F32 ? ((const float *)e.bias)[n] : ldf((const __nv_bfloat16 *)e.bias + n);
    v = e.epi == MTP_EPI_BIAS_SOFTPLUS ? softplus_f(v + b) : v + b;
  }
  if (e.c_dtype == MTP_F32) ((float *)e.C)[(size_t)m * e.ldc + n] = v;
  else ((__nv_bfloat16 *)e.C)[(size_t)m * e.ldc + n] = __float2bfloat16_rn(v);
}

// ----------------------------------------------------------------- SIMT tiled GEMM
template <typename T>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const T *__restrict__ A, const T *__restrict__ B, int M, int N,
                                                        int K, int lda, int ldb, EpiArgs e) {
  MTP_PDL_WAIT();
  MTP_PDL_TRIGGER();
  __shared__ float As[16][68];
  __shared__ float Bs[16][68];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int el = tid + i * 256, r = el >> 4, kk = el & 15;
      As[kk][r] = (m0 + r < M && k0 + kk < K) ? ldf(A + (size_t)(m0 + r) * lda + k0 + kk) : 0.f;
      Bs[kk][r] = (n0 + r < N && k0 + kk < K) ? ldf(B + (size_t)(n0 + r) * ldb + k0 + kk) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) { a[i] = As[kk][ty * 4 + i]; b[i] = Bs[kk][tx * 4 + i]; }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int m = m0 + ty * 4 + i, n = n0 + tx * 4 + j;
      if (m < M && n < N) epi_store(e, m, n, acc[i][j]);
    }
}

// ----------------------------------------------------------------- small-M GEMV
template <typename T> struct Vec8;
template <> struct Vec8<__nv_bfloat16> {
  static __device__ __forceinline__ void load(const __nv_bfloat16 *p, float (&v)[8]) {
    const uint4 u = __ldg(reinterpret_cast<const uint4 *>(p));
    const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
};
template <> struct Vec8<float> {
  static __device__ __forceinline__ void load(const float *p, float (&v)[8]) {
    const float4 a = __ldg(reinterpret_cast<const float4 *>(p));
    const float4 b = __ldg(reinterpret_cast<const float4 *>(p + 4));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
};

template <typename T>
__device__ __forceinline__ void load8(const T *p, int k, int K, bool vec, float (&v)[8]) {
  if (vec && k + 8 <= K) {
    Vec8<T>::load(p + k, v);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = (k + i < K) ? ldf(p + k + i) : 0.f;
  }
}

template <typename T, int MT, int ROWS>
__global__ void __launch_bounds__(256) gemv_kernel(const T *__restrict__ X, int ldx, const T *__restrict__ W, int ldw,
                                                   int M, int N, int K, bool vec, EpiArgs e) {
  MTP_PDL_WAIT();
  MTP_PDL_TRIGGER();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_base = (blockIdx.x * (blockDim.x >> 5) + warp) * ROWS;
  const int m0 = blockIdx.y * MT;
  if (n_base >= N) return;
  float acc[ROWS][MT];
#pragma unroll
  for (int r = 0; r < ROWS; ++r)
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[r][m] = 0.f;
  constexpr int U = MT <= 2 ? 4 : 1;  // k-steps of weight loads in flight per lane
  for (int k0 = lane * 8; k0 < K; k0 += 256 * U) {
    float w[U][ROWS][8];
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int r = 0; r < ROWS; ++r) {
        const int k = k0 + 256 * u;
        if (n_base + r < N && k < K) load8(W + (size_t)(n_base + r) * ldw, k, K, vec, w[u][r]);
        else {
#pragma unroll
          for (int i = 0; i < 8; ++i) w[u][r][i] = 0.f;
        }
      }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int k = k0 + 256 * u;
      if (k >= K) break;
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        if (m0 + m >= M) break;
        float x[8];
        load8(X + (size_t)(m0 + m) * ldx, k, K, vec, x);
#pragma unroll
        for (int r = 0; r < ROWS; ++r)
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[r][m] = fmaf(w[u][r][i], x[i], acc[r][m]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < ROWS; ++r)
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      float v = acc[r][m];
#pragma unroll
      for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      acc[r][m] = v;
    }
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
#pragma unroll
      for (int m = 0; m < MT; ++m)
        if (n_base + r < N && m0 + m < M) epi_store(e, m0 + m, n_base + r, acc[r][m]);
  }
}

// Block-split-K GEMV for small N: a CTA of 256 threads owns RB output rows and
// all MT tokens; its threads stride over K (8 elements each, 16-byte loads, U
// loads in flight), then the partial sums are reduced across the 8 warps in
// shared memory in a fixed order.
template <typename T, int MT, int RB>
__global__ void __launch_bounds__(256) gemv_splitk_kernel(const T *__restrict__ X, int ldx, const T *__restrict__ W,
                                                          int ldw, int M, int N, int K, bool vec, EpiArgs e) {
  MTP_PDL_WAIT();
  MTP_PDL_TRIGGER();
  __shared__ float red[8][RB][MT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * RB, m0 = blockIdx.y * MT;
  float acc[RB][MT];
#pragma unroll
  for (int r = 0; r < RB; ++r)
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[r][m] = 0.f;
  constexpr int U = 2;
  for (int k0 = threadIdx.x * 8; k0 < K; k0 += 2048 * U) {
    float w[U][RB][8];
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        const int k = k0 + 2048 * u;
        if (n0 + r < N && k < K) load8(W + (size_t)(n0 + r) * ldw, k, K, vec, w[u][r]);
        else {
#pragma unroll
          for (int i = 0; i < 8; ++i) w[u][r][i] = 0.f;
        }
      }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int k = k0 + 2048 * u;
      if (k >= K) break;
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        if (m0 + m >= M) break;
        float x[8];
        load8(X + (size_t)(m0 + m) * ldx, k, K, vec, x);
#pragma unroll
        for (int r = 0; r < RB; ++r)
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[r][m] = fmaf(w[u][r][i], x[i], acc[r][m]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RB; ++r)
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      float v = acc[r][m];
#pragma unroll
      for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) red[warp][r][m] = v;
    }
  __syncthreads();
  if (threadIdx.x < RB * MT) {
    const int r = threadIdx.x / MT, m = threadIdx.x % MT;
    float v = 0.f;
#pragma unroll
    for (int wi = 0; wi < 8; ++wi) v += red[wi][r][m];
    if (n0 + r < N && m0 + m < M) epi_store(e, m0 + m, n0 + r, v);
  }
}

// The GEMV variant for [M, N] x K: K split over a CTA's threads for small N (more CTAs
// than rows of W otherwise), one warp per row of W else.  The two sum K in different orders.
static bool gemv_splits_k(int M, int N, int K) { return N <= 4096 && K >= 512 && M <= 8; }

template <typename T>
static int launch_gemv(const T *X, int ldx, const T *W, int ldw, int M, int N, int K, EpiArgs e, cudaStream_t s,
                       int split = -1) {
  constexpr int ROWS = 2;
  const bool vec = aligned16(X) && aligned16(W) && (ldx % 8 == 0) && (ldw % 8 == 0);
  if (split < 0) split = gemv_splits_k(M, N, K) ? 1 : 0;
  if (split) {  // small N: every CTA splits K over its 256 threads
    constexpr int RB = 2;
    dim3 g(ceil_div(N, RB));
    if (M <= 1) launch_pdl(gemv_splitk_kernel<T, 1, RB>, dim3(g), dim3(256), 0, s, X, ldx, W, ldw, M, N, K, vec, e);
    else if (M <= 2) launch_pdl(gemv_splitk_kernel<T, 2, RB>, dim3(g), dim3(256), 0, s, X, ldx, W, ldw, M, N, K, vec, e);
    else if (M <= 4) launch_pdl(gemv_splitk_kernel<T, 4, RB>, dim3(g), dim3(256), 0, s, X, ldx, W, ldw, M, N, K, vec, e);
    else launch_pdl(gemv_splitk_kernel<T, 8, RB>, dim3(g), dim3(256), 0, s, X, ldx, W, ldw, M, N, K, vec, e);
    return check_launch("gemv_splitk");
  }
  const int rows_per_block = 8 * ROWS;
  dim3 grid(ceil_div(N, rows_per_block));
  if (M <= 1) { grid.y = 1; launch_pdl(gemv_kernel<T, 1, ROWS>, dim3(grid), dim3(256), 0, s, X, ldx, W, ldw, M, N, K, vec, e); }
  else if (M <= 2) { grid.y = 1; launch_pdl(gemv_kernel<T, 2, ROWS>, dim3(grid), dim3(256), 0, s, X, ldx, W, ldw, M, N, K, vec, e); }
  else if (M <= 4) { grid.y = 1; launch_pdl(gemv_kernel<T, 4, ROWS>, dim3(grid), dim3(256), 0, s, X, ldx, W, ldw, M, N, K, vec, e); }
  else { grid.y = ceil_div(M, 8); launch_pdl(gemv_kernel<T, 8, ROWS>, dim3(grid), dim3(256), 0, s, X, ldx, W, ldw, M, N, K, vec, e); }
  return check_launch("gemv");
}

// Columns [col0, col0 + cols) of C = A x B^T for a B of N_full rows, computed by the
// kernel (and so with the per-element summation order) that mtp_gemm picks for the whole
// [M, N_full] product: the vocabulary-parallel lm_head gives the same bits as the
// replicated one.  B and C are the full matrices; C's other columns are not touched.
int gemm_cols_as_full(const void *A, const void *B, void *C, int M, int N_full, int col0, int cols, int K, int lda,
                      int ldb, int ldc, int dtype, cudaStream_t s) {
  MTP_REQUIRE(A && B && C && M >= 0 && K > 0 && col0 >= 0 && cols > 0 && col0 + cols <= N_full, "bad arguments");
  MTP_REQUIRE(dtype == MTP_F32 || dtype == MTP_BF16, "dtype must be F32 or BF16");
  if (M == 0) return MTP_OK;
  const size_t es = dtype == MTP_F32 ? 4 : 2;
  const void *Bs = (const char *)B + (size_t)col0 * ldb * es;
  void *Cs = (char *)C + (size_t)col0 * es;
  EpiArgs e{Cs, ldc, dtype, MTP_EPI_STORE, nullptr, 0};
  if (dtype == MTP_BF16 && M > 16 && gemm_tc_eligible(A, B, M, N_full, K, lda, ldb)) {
    MTP_REQUIRE(aligned16(Bs), "vocabulary shard of B not 16-byte aligned");
    return gemm_tc(A, Bs, Cs, M, cols, K, lda, ldb, ldc, dtype, MTP_EPI_STORE, nullptr, 0, s);
  }
  if (M <= 64) {
    const int split = gemv_splits_k(M, N_full, K) ? 1 : 0;
    if (dtype == MTP_F32) return launch_gemv((const float *)A, lda, (const float *)Bs, ldb, M, cols, K, e, s, split);
    return launch_gemv((const __nv_bfloat16 *)A, lda, (const __nv_bfloat16 *)Bs, ldb, M, cols, K, e, s, split);
  }
  dim3 grid(ceil_div(cols, 64), ceil_div(M, 64));
  if (dtype == MTP_F32)
    launch_pdl(gemm_simt_kernel<float>, dim3(grid), dim3(256), 0, s, (const float *)A, (const float *)Bs, M, cols, K,
               lda, ldb, e);
  else
    launch_pdl(gemm_simt_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, s, (const __nv_bfloat16 *)A,
               (const __nv_bfloat16 *)Bs, M, cols, K, lda, ldb, e);
  return check_launch("gemm_simt");
}

}  // namespace mtp

using namespace mtp;

extern "C" {

int mtp_gemm_ex(const void *A, const void *B, void *C, int M, int N, int K, int lda, int ldb, int ldc, int ab_dtype,
                int c_dtype, int epilogue, const void *bias, int bias_dtype, int algo, void *stream) {
  MTP_REQUIRE(A && B && C, "null pointer");
  MTP_REQUIRE(M >= 0 && N > 0 && K > 0, "bad sizes");
  MTP_REQUIRE(lda >= K && ldb >= K && ldc >= N, "leading dimensions too small");
  MTP_REQUIRE(c_dtype == MTP_F32 || c_dtype == MTP_BF16, "C must be F32 or BF16");
  MTP_REQUIRE(ab_dtype == MTP_F32 || ab_dtype == MTP_BF16, "A/B must be F32 or BF16");
  MTP_REQUIRE(epilogue == MTP_EPI_STORE || ((epilogue == MTP_EPI_BIAS_SOFTPLUS || epilogue == MTP_EPI_BIAS) && bias),
              "bad epilogue");
  MTP_REQUIRE(!bias || bias_dtype == MTP_F32 || bias_dtype == MTP_BF16, "bias must be F32 or BF16");
  if (M == 0) return MTP_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if (algo == MTP_GEMM_AUTO) {
    if (ab_dtype == MTP_BF16 && M > 16 && gemm_tc_eligible(A, B, M, N, K, lda, ldb)) algo = MTP_GEMM_TCGEN05;
    else if (M <= 64) algo = MTP_GEMM_GEMV;
    else algo = MTP_GEMM_SIMT;
  }
  EpiArgs e{C, ldc, c_dtype, epilogue, bias, bias_dtype};
  if (algo == MTP_GEMM_TCGEN05) {
    MTP_REQUIRE(ab_dtype == MTP_BF16, "the tcgen05 GEMM takes bf16 operands");
    return gemm_tc(A, B, C, M, N, K, lda, ldb, ldc, c_dtype, epilogue, bias, bias_dtype, s);
  }
  if (algo == MTP_GEMM_GEMV) {
    if (ab_dtype == MTP_F32) return launch_gemv((const float *)A, lda, (const float *)B, ldb, M, N, K, e, s);
    return launch_gemv((const __nv_bfloat16 *)A, lda, (const __nv_bfloat16 *)B, ldb, M, N, K, e, s);
  }
  if (algo == MTP_GEMM_SIMT) {
    dim3 grid(ceil_div(N, 64), ceil_div(M, 64));
    if (ab_dtype == MTP_F32)
      launch_pdl(gemm_simt_kernel<float>, dim3(grid), dim3(256), 0, s, (const float *)A, (const float *)B, M, N, K, lda, ldb, e);
    else
      launch_pdl(gemm_simt_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, s, (const __nv_bfloat16 *)A, (const __nv_bfloat16 *)B, M, N,
                                                           K, lda, ldb, e);
    return check_launch("gemm_simt");
  }
  return fail(MTP_ERR_ARG, "unknown GEMM algorithm");
}

int mtp_gemm(const void *A, const void *B, void *C, int M, int N, int K, int lda, int ldb, int ldc, int ab_dtype,
             int c_dtype, int epilogue, const void *bias, int bias_dtype, void *stream) {
  return mtp_gemm_ex(A, B, C, M, N, K, lda, ldb, ldc, ab_dtype, c_dtype, epilogue, bias, bias_dtype, MTP_GEMM_AUTO,
                     stream);
}

}  // extern "C"
