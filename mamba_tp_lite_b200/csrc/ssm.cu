// Selective-scan kernels: conv1d+SiLU, fused prefill scan, single-token step.
//
// Math (per batch b, channel c, state n; A = -exp(A_log)):
//   xc_t  = silu(conv_b + sum_j conv_w[j] * xpad[t + j])      (causal, K taps)
//   h_t   = exp(dt_t * A_n) * h_{t-1} + (dt_t * B_t[n]) * xc_t
//   y_t   = (sum_n C_t[n] * h_t[n] + D * xc_t) * silu(z_t)
// restating mamba_lite/tp_model.py:93-129 (prefill) and :145-173 (step).
#include "common.cuh"

namespace mtp {

constexpr float kLog2e = 1.4426950408889634f;

// exp(x) for x = dt*A <= 0 through the hardware base-2 exponential: exp(x) = 2^(x*log2 e).
__device__ __forceinline__ float ex2_hw(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void cp_async4(void *smem, const void *gmem) {
  uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int NG> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(NG) : "memory");
}

// ----------------------------------------------------------------- conv1d + SiLU
// One thread per (channel, run of TT consecutive positions); the K-1 input
// window slides in registers.
template <typename T, int K, int TT>
__global__ void conv1d_silu_kernel(const T *__restrict__ xz, int ld_xz, const T *__restrict__ w,
                                   const T *__restrict__ bias, const T *__restrict__ hist, T *__restrict__ xc,
                                   int ld_xc, int L, int Es) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int t0 = blockIdx.y * TT;
  const int b = blockIdx.z;
  if (c >= Es) return;
  float wk[K];
#pragma unroll
  for (int j = 0; j < K; ++j) wk[j] = ldf(w + (size_t)c * K + j);
  const float bc = bias ? ldf(bias + c) : 0.f;
  float win[K - 1];
#pragma unroll
  for (int j = 0; j < K - 1; ++j) {
    const int t = t0 - (K - 1) + j;  // input position
    float v = 0.f;
    if (t >= 0) v = ldf(xz + (size_t)(b * (size_t)L + t) * ld_xz + c);
    else if (hist) v = ldf(hist + ((size_t)b * Es + c) * (K - 1) + (K - 1 + t));
    win[j] = v;
  }
#pragma unroll
  for (int i = 0; i < TT; ++i) {
    const int t = t0 + i;
    if (t >= L) break;
    const float xv = ldf(xz + (size_t)(b * (size_t)L + t) * ld_xz + c);
    float acc = bc;
#pragma unroll
    for (int j = 0; j < K - 1; ++j) acc += wk[j] * win[j];
    acc += wk[K - 1] * xv;
#pragma unroll
    for (int j = 0; j < K - 2; ++j) win[j] = win[j + 1];
    win[K - 2] = xv;
    stf(xc + (size_t)(b * (size_t)L + t) * ld_xc + c, silu_f(acc));
  }
}

// ----------------------------------------------------------------- fused prefill scan
// CTA = (channel block of CB channels, one sequence b); TPC threads share one
// channel, each holding N/TPC states in registers.  The sequence is walked in
// chunks of TL positions staged in shared memory by cp.async (double buffer):
// raw x, z, dt for the block's channels and B|C (shared by all channels).
template <typename T, int N, int TPC, int CB, int TL>
struct ScanSmem {
  T x[2][TL][CB];
  T z[2][TL][CB];
  float dt[2][TL][CB];
  float bc[2][TL][2 * N];
  float y[TL][CB];
};

template <typename T, int N, int TPC, int CB, int TL, int K>
__global__ void __launch_bounds__(CB *TPC) scan_prefill_kernel(
    const T *__restrict__ xz, int ld_xz, const float *__restrict__ dtp, int ld_dt, const float *__restrict__ bcp,
    int ld_bc, const T *__restrict__ A_log, const T *__restrict__ Dp, const T *__restrict__ conv_w,
    const T *__restrict__ conv_b, const T *conv_init, const float *ssm_init, T *__restrict__ y, int ld_y,
    T *conv_final, float *ssm_final, int L, int Es) {
  constexpr int NS = N / TPC;
  constexpr int NT = CB * TPC;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  auto &sm = *reinterpret_cast<ScanSmem<T, N, TPC, CB, TL> *>(smem_raw);

  const int b = blockIdx.y;
  const int c0 = blockIdx.x * CB;
  const int cl = threadIdx.x / TPC;
  const int sub = threadIdx.x % TPC;
  const int c = c0 + cl;
  const bool live = c < Es;
  const int ncb = min(CB, Es - c0);  // live channels in this block
  const size_t row0 = (size_t)b * L;

  // per-thread constants
  float A2[NS], h[NS];
  float wk[K], win[K - 1];
  float Dv = 0.f, cbias = 0.f;
#pragma unroll
  for (int i = 0; i < NS; ++i) {
    const int n = sub * NS + i;
    A2[i] = live ? -expf(ldf(A_log + (size_t)c * N + n)) * kLog2e : 0.f;
    h[i] = (live && ssm_init) ? ssm_init[((size_t)b * Es + c) * N + n] : 0.f;
  }
#pragma unroll
  for (int j = 0; j < K; ++j) wk[j] = live ? ldf(conv_w + (size_t)c * K + j) : 0.f;
#pragma unroll
  for (int j = 0; j < K - 1; ++j)
    win[j] = (live && conv_init) ? ldf(conv_init + ((size_t)b * Es + c) * (K - 1) + j) : 0.f;
  if (live) {
    Dv = ldf(Dp + c);
    cbias = conv_b ? ldf(conv_b + c) : 0.f;
  }

  // cooperative async load of chunk k into buffer buf (4-byte granules)
  auto load_chunk = [&](int k, int buf) {
    const int t0 = k * TL;
    const int tl = min(TL, L - t0);
    constexpr int EPW = 4 / sizeof(T);  // elements per 4-byte word for x / z
    const int wpr = (ncb + EPW - 1) / EPW;  // words per row
    for (int i = threadIdx.x; i < tl * wpr; i += NT) {
      const int tt = i / wpr, wi = i % wpr;
      const size_t r = row0 + t0 + tt;
      cp_async4(&sm.x[buf][tt][wi * EPW], xz + r * ld_xz + c0 + wi * EPW);
      cp_async4(&sm.z[buf][tt][wi * EPW], xz + r * ld_xz + Es + c0 + wi * EPW);
    }
    for (int i = threadIdx.x; i < tl * ncb; i += NT) {
      const int tt = i / ncb, ci = i % ncb;
      cp_async4(&sm.dt[buf][tt][ci], dtp + (row0 + t0 + tt) * ld_dt + c0 + ci);
    }
    for (int i = threadIdx.x; i < tl * 2 * N; i += NT) {
      const int tt = i / (2 * N), j = i % (2 * N);
      cp_async4(&sm.bc[buf][tt][j], bcp + (row0 + t0 + tt) * ld_bc + j);
    }
    cp_async_commit();
  };

  const int nchunks = (L + TL - 1) / TL;
  load_chunk(0, 0);
  for (int k = 0; k < nchunks; ++k) {
    const int buf = k & 1;
    if (k + 1 < nchunks) {
      load_chunk(k + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int t0 = k * TL;
    const int tl = min(TL, L - t0);
    // every lane runs the loop (the group shuffle needs all 32); lanes past the
    // last channel read in-bounds shared memory and store nothing
    {
      for (int tt = 0; tt < tl; ++tt) {
        const float xv = ldf(&sm.x[buf][tt][cl]);
        float acc = cbias;
#pragma unroll
        for (int j = 0; j < K - 1; ++j) acc += wk[j] * win[j];
        acc += wk[K - 1] * xv;
#pragma unroll
        for (int j = 0; j < K - 2; ++j) win[j] = win[j + 1];
        win[K - 2] = xv;
        const float xc = silu_f(acc);
        const float dt = sm.dt[buf][tt][cl];
        const float *bcr = sm.bc[buf][tt];
        float yv = 0.f;
#pragma unroll
        for (int i = 0; i < NS; ++i) {
          const int n = sub * NS + i;
          const float dA = ex2_hw(dt * A2[i]);
          const float dBx = (dt * bcr[n]) * xc;
          h[i] = fmaf(dA, h[i], dBx);
          yv = fmaf(bcr[N + n], h[i], yv);
        }
#pragma unroll
        for (int o = 1; o < TPC; o <<= 1) yv += __shfl_xor_sync(0xffffffffu, yv, o);
        if (sub == 0 && live) {
          const float zv = ldf(&sm.z[buf][tt][cl]);
          sm.y[tt][cl] = (yv + Dv * xc) * silu_f(zv);
        }
      }
    }
    __syncthreads();
    // coalesced store of the chunk's y
    for (int i = threadIdx.x; i < tl * ncb; i += NT) {
      const int tt = i / ncb, ci = i % ncb;
      stf(y + (row0 + t0 + tt) * ld_y + c0 + ci, sm.y[tt][ci]);
    }
    // buffer `buf` is refilled by the next iteration's prefetch only after this barrier
    __syncthreads();
  }
  if (live) {
#pragma unroll
    for (int i = 0; i < NS; ++i) ssm_final[((size_t)b * Es + c) * N + sub * NS + i] = h[i];
    if (sub == 0) {
#pragma unroll
      for (int j = 0; j < K - 1; ++j) stf(conv_final + ((size_t)b * Es + c) * (K - 1) + j, win[j]);
    }
  }
}

// ----------------------------------------------------------------- single-token step
// CTA = CB channels x all B sequences.  dt_proj rows of the block and the
// dt_low vectors are staged in shared memory; then one thread per (b, c)
// does conv shift, dt, state update and output, all in place.
template <typename T, int N, int K, int CB>
__global__ void __launch_bounds__(256) step_kernel(const T *__restrict__ xz, int ld_xz, const T *__restrict__ dt_low,
                                                   int ld_dl, const T *__restrict__ W_dt, const T *__restrict__ b_dt,
                                                   const float *__restrict__ bcp, int ld_bc, const T *__restrict__ A_log,
                                                   const T *__restrict__ Dp, const T *__restrict__ conv_w,
                                                   const T *__restrict__ conv_b, T *conv_state, float *ssm_state,
                                                   T *__restrict__ y, int ld_y, int B, int Es, int R) {
  extern __shared__ __align__(16) float ssm_sm[];
  const int RP = R + 1;  // padded row stride against bank conflicts
  float *wdt = ssm_sm;               // [CB][RP]
  float *dl = ssm_sm + CB * RP;      // [B][R]
  const int c0 = blockIdx.x * CB;
  const int ncb = min(CB, Es - c0);
  for (int i = threadIdx.x; i < ncb * R; i += blockDim.x) {
    const int cc = i / R, r = i % R;
    wdt[cc * RP + r] = ldf(W_dt + (size_t)(c0 + cc) * R + r);
  }
  for (int i = threadIdx.x; i < B * R; i += blockDim.x) {
    const int bb = i / R, r = i % R;
    dl[bb * R + r] = ldf(dt_low + (size_t)bb * ld_dl + r);
  }
  __syncthreads();
  for (int p = threadIdx.x; p < B * ncb; p += blockDim.x) {
    const int bb = p / ncb, cc = p % ncb, c = c0 + cc;
    // dt_proj + bias + softplus (tp_model.py:162-163)
    float s = 0.f;
    const float *wr = wdt + cc * RP;
    const float *xr = dl + bb * R;
    for (int r = 0; r < R; ++r) s = fmaf(xr[r], wr[r], s);
    const float dt = softplus_f(s + ldf(b_dt + c));
    // conv over [history | x] then shift (tp_model.py:145-157)
    T *cs = conv_state + ((size_t)bb * Es + c) * (K - 1);
    const float xv = ldf(xz + (size_t)bb * ld_xz + c);
    float acc = conv_b ? ldf(conv_b + c) : 0.f;
    float hist[K - 1];
#pragma unroll
    for (int j = 0; j < K - 1; ++j) {
      hist[j] = ldf(cs + j);
      acc += ldf(conv_w + (size_t)c * K + j) * hist[j];
    }
    acc += ldf(conv_w + (size_t)c * K + K - 1) * xv;
#pragma unroll
    for (int j = 0; j < K - 2; ++j) stf(cs + j, hist[j + 1]);
    stf(cs + K - 2, xv);
    const float xc = silu_f(acc);
    // state update and output (tp_model.py:165-173)
    float *hs = ssm_state + ((size_t)bb * Es + c) * N;
    const float *bcr = bcp + (size_t)bb * ld_bc;
    float yv = 0.f;
#pragma unroll
    for (int n = 0; n < N; ++n) {
      const float a2 = -expf(ldf(A_log + (size_t)c * N + n)) * kLog2e;
      const float dA = ex2_hw(dt * a2);
      const float hv = fmaf(dA, hs[n], (dt * bcr[n]) * xc);
      hs[n] = hv;
      yv = fmaf(bcr[N + n], hv, yv);
    }
    const float zv = ldf(xz + (size_t)bb * ld_xz + Es + c);
    stf(y + (size_t)bb * ld_y + c, (yv + ldf(Dp + c) * xc) * silu_f(zv));
  }
}

template <typename T, int N, int TPC>
static int launch_scan(const void *xz, int ld_xz, const float *dt, int ld_dt, const float *bc, int ld_bc,
                       const void *A_log, const void *Dp, const void *conv_w, const void *conv_b,
                       const void *conv_init, const float *ssm_init, void *y, int ld_y, void *conv_final,
                       float *ssm_final, int B, int L, int Es, cudaStream_t s) {
  constexpr int CB = 64, TL = 32, K = 4;
  using S = ScanSmem<T, N, TPC, CB, TL>;
  auto kern = scan_prefill_kernel<T, N, TPC, CB, TL, K>;
  static bool attr_set = false;  // per template instance
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(S)) != cudaSuccess)
      return check_launch("scan_prefill attr");
    attr_set = true;
  }
  dim3 grid((Es + CB - 1) / CB, B);
  kern<<<grid, CB * TPC, sizeof(S), s>>>((const T *)xz, ld_xz, dt, ld_dt, bc, ld_bc, (const T *)A_log,
                                          (const T *)Dp, (const T *)conv_w, (const T *)conv_b, (const T *)conv_init,
                                          ssm_init, (T *)y, ld_y, (T *)conv_final, ssm_final, L, Es);
  return check_launch("scan_prefill");
}

}  // namespace mtp

using namespace mtp;

extern "C" {

int mtp_conv1d_silu(const void *xz, int ld_xz, const void *conv_w, const void *conv_b, const void *hist, void *xc,
                    int ld_xc, int B, int L, int Es, int K, int dtype, void *stream) {
  MTP_REQUIRE(xz && conv_w && xc && B >= 0 && L >= 0 && Es > 0, "bad arguments");
  MTP_REQUIRE(K == 4, "only d_conv == 4 is built");
  MTP_REQUIRE(ld_xz >= 2 * Es && ld_xc >= Es, "leading dimensions too small");
  if (B == 0 || L == 0) return MTP_OK;
  constexpr int TT = 8;
  dim3 grid((Es + 127) / 128, (L + TT - 1) / TT, B);
  cudaStream_t s = (cudaStream_t)stream;
  MTP_DISPATCH_FB(dtype, T,
      conv1d_silu_kernel<T, 4, TT><<<grid, 128, 0, s>>>((const T *)xz, ld_xz, (const T *)conv_w,
                                                         (const T *)conv_b, (const T *)hist, (T *)xc, ld_xc, L, Es));
  return check_launch("conv1d_silu");
}

int mtp_scan_prefill(const void *xz, int ld_xz, const float *dt, int ld_dt, const float *bc, int ld_bc,
                     const void *A_log, const void *Dp, const void *conv_w, const void *conv_b, const void *conv_init,
                     const float *ssm_init, void *y, int ld_y, void *conv_final, float *ssm_final, int B, int L,
                     int Es, int N, int K, int dtype, void *stream) {
  MTP_REQUIRE(xz && dt && bc && A_log && Dp && conv_w && y && conv_final && ssm_final, "null pointer");
  MTP_REQUIRE(B >= 0 && L >= 0 && Es > 0, "bad sizes");
  MTP_REQUIRE(K == 4, "only d_conv == 4 is built");
  MTP_REQUIRE(N == 16 || N == 8, "d_state must be 8 or 16");
  MTP_REQUIRE(ld_xz >= 2 * Es && ld_dt >= Es && ld_bc >= 2 * N && ld_y >= Es, "leading dimensions too small");
  const size_t es = dtype == MTP_F32 ? 4 : 2;
  // 4-byte cp.async granules: x/z words must be 4-byte aligned
  MTP_REQUIRE(aligned(xz, 4) && aligned(dt, 4) && aligned(bc, 4), "inputs must be 4-byte aligned");
  MTP_REQUIRE(es == 4 || (ld_xz % 2 == 0 && Es % 2 == 0), "bf16 x|z rows need even Es and ld_xz");
  if (B == 0 || L == 0) return MTP_OK;
  cudaStream_t s = (cudaStream_t)stream;
  // threads per channel: enough resident warps at small channel counts
  const long pairs = (long)B * Es;
  const int sms = num_sms();
  const int tpc = pairs >= (long)sms * 1024 ? 1 : (pairs >= (long)sms * 384 ? 2 : 4);
#define MTP_SCAN_CASE(TT, NN, TP)                                                                          \
  return launch_scan<TT, NN, TP>(xz, ld_xz, dt, ld_dt, bc, ld_bc, A_log, Dp, conv_w, conv_b, conv_init,   \
                                 ssm_init, y, ld_y, conv_final, ssm_final, B, L, Es, s)
  if (dtype == MTP_F32) {
    if (N == 16) { if (tpc == 1) MTP_SCAN_CASE(float, 16, 1); if (tpc == 2) MTP_SCAN_CASE(float, 16, 2); MTP_SCAN_CASE(float, 16, 4); }
    MTP_SCAN_CASE(float, 8, 2);
  } else if (dtype == MTP_BF16) {
    if (N == 16) { if (tpc == 1) MTP_SCAN_CASE(__nv_bfloat16, 16, 1); if (tpc == 2) MTP_SCAN_CASE(__nv_bfloat16, 16, 2); MTP_SCAN_CASE(__nv_bfloat16, 16, 4); }
    MTP_SCAN_CASE(__nv_bfloat16, 8, 2);
  }
#undef MTP_SCAN_CASE
  return fail(MTP_ERR_UNSUPPORTED, "scan_prefill: dtype must be F32 or BF16");
}

int mtp_step(const void *xz, int ld_xz, const void *dt_low, int ld_dl, const void *W_dt, const void *b_dt,
             const float *bc, int ld_bc, const void *A_log, const void *Dp, const void *conv_w, const void *conv_b,
             void *conv_state, float *ssm_state, void *y, int ld_y, int B, int Es, int N, int R, int K, int dtype,
             void *stream) {
  MTP_REQUIRE(xz && dt_low && W_dt && b_dt && bc && A_log && Dp && conv_w && conv_state && ssm_state && y,
              "null pointer");
  MTP_REQUIRE(K == 4, "only d_conv == 4 is built");
  MTP_REQUIRE(N == 16 || N == 8, "d_state must be 8 or 16");
  MTP_REQUIRE(B >= 0 && B <= 256 && Es > 0 && R > 0 && R <= 512, "bad sizes");
  if (B == 0) return MTP_OK;
  constexpr int CB = 32;
  const size_t smem = ((size_t)CB * (R + 1) + (size_t)B * R) * sizeof(float);
  MTP_REQUIRE(smem <= 200 * 1024, "batch x dt_rank too large for the step kernel");
  cudaStream_t s = (cudaStream_t)stream;
  dim3 grid((Es + CB - 1) / CB);
#define MTP_STEP_CASE(TT, NN)                                                                               \
  do {                                                                                                     \
    auto kern = step_kernel<TT, NN, 4, CB>;                                                                \
    static bool attr_set = false;                                                                          \
    if (!attr_set) {                                                                                       \
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);                 \
      attr_set = true;                                                                                     \
    }                                                                                                      \
    kern<<<grid, 256, smem, s>>>((const TT *)xz, ld_xz, (const TT *)dt_low, ld_dl, (const TT *)W_dt,       \
                                 (const TT *)b_dt, bc, ld_bc, (const TT *)A_log, (const TT *)Dp,          \
                                 (const TT *)conv_w, (const TT *)conv_b, (TT *)conv_state, ssm_state,     \
                                 (TT *)y, ld_y, B, Es, R);                                                 \
    return check_launch("step");                                                                           \
  } while (0)
  if (dtype == MTP_F32) { if (N == 16) MTP_STEP_CASE(float, 16); MTP_STEP_CASE(float, 8); }
  if (dtype == MTP_BF16) { if (N == 16) MTP_STEP_CASE(__nv_bfloat16, 16); MTP_STEP_CASE(__nv_bfloat16, 8); }
#undef MTP_STEP_CASE
  return fail(MTP_ERR_UNSUPPORTED, "step: dtype must be F32 or BF16");
}

}  // extern "C"
