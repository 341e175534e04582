// Selective-scan kernels: conv1d+SiLU, fused prefill scan, single-token step.
//
// Math (per batch b, channel c, state n; A = -exp(A_log)):
//   xc_t  = silu(conv_b + sum_j conv_w[j] * xpad[t + j])      (causal, K taps)
//   h_t   = exp(dt_t * A_n) * h_{t-1} + (dt_t * B_t[n]) * xc_t
//   y_t   = (sum_n C_t[n] * h_t[n] + D * xc_t) * silu(z_t)
// restating mamba_lite/tp_model.py:93-129 (prefill) and :145-173 (step).
#include <cstdlib>
#include <type_traits>
#include <cstring>
#include "common.cuh"
#include "tc_common.cuh"

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
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
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
  MTP_PDL_WAIT();
  MTP_PDL_TRIGGER();
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

// Vectorised variant: one thread per (16-byte group of VEC channels, run of TT
// positions); loads and stores are 16 bytes wide.  Needs Es % VEC == 0 and
// 16-byte aligned rows.
template <typename T> struct Pack16;
template <> struct Pack16<__nv_bfloat16> {
  static constexpr int V = 8;
  static __device__ __forceinline__ void load(const __nv_bfloat16 *p, float (&v)[8]) {
    const uint4 u = *reinterpret_cast<const uint4 *>(p);
    const __nv_bfloat162 *h2 = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h2[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
  static __device__ __forceinline__ void store(__nv_bfloat16 *p, const float (&v)[8]) {
    uint4 u;
    __nv_bfloat162 *h2 = reinterpret_cast<__nv_bfloat162 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h2[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4 *>(p) = u;
  }
};
template <> struct Pack16<float> {
  static constexpr int V = 4;
  static __device__ __forceinline__ void load(const float *p, float (&v)[4]) {
    const float4 f = *reinterpret_cast<const float4 *>(p);
    v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
  }
  static __device__ __forceinline__ void store(float *p, const float (&v)[4]) {
    *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
};

template <typename T, int K, int TT>
__global__ void conv1d_silu_vec_kernel(const T *__restrict__ xz, int ld_xz, const T *__restrict__ w,
                                       const T *__restrict__ bias, const T *__restrict__ hist, T *__restrict__ xc,
                                       int ld_xc, int L, int Es, bool wvec) {
  MTP_PDL_WAIT();
  MTP_PDL_TRIGGER();
  constexpr int V = Pack16<T>::V;
  static_assert(V * K * sizeof(T) == 64, "a group's taps are four 16-byte words");
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * V;
  const int t0 = blockIdx.y * TT;
  const int b = blockIdx.z;
  if (c >= Es) return;
  float wk[V][K], bc[V], win[V][K - 1];
  if (wvec) {  // the group's V x K taps and V biases as 16-byte loads
    T tw[V * K], tb[V];
#pragma unroll
    for (int q = 0; q < 4; ++q) reinterpret_cast<uint4 *>(tw)[q] = __ldg(reinterpret_cast<const uint4 *>(w + (size_t)c * K) + q);
    if (bias) *reinterpret_cast<uint4 *>(tb) = __ldg(reinterpret_cast<const uint4 *>(bias + c));
#pragma unroll
    for (int u = 0; u < V; ++u) {
#pragma unroll
      for (int j = 0; j < K; ++j) wk[u][j] = ldf(&tw[u * K + j]);
      bc[u] = bias ? ldf(&tb[u]) : 0.f;
    }
  } else {
#pragma unroll
    for (int u = 0; u < V; ++u) {
#pragma unroll
      for (int j = 0; j < K; ++j) wk[u][j] = ldf(w + (size_t)(c + u) * K + j);
      bc[u] = bias ? ldf(bias + c + u) : 0.f;
    }
  }
#pragma unroll
  for (int j = 0; j < K - 1; ++j) {
    const int t = t0 - (K - 1) + j;
    if (t >= 0) {
      float v[V];
      Pack16<T>::load(xz + (size_t)(b * (size_t)L + t) * ld_xz + c, v);
#pragma unroll
      for (int u = 0; u < V; ++u) win[u][j] = v[u];
    } else {
#pragma unroll
      for (int u = 0; u < V; ++u) win[u][j] = hist ? ldf(hist + ((size_t)b * Es + c + u) * (K - 1) + (K - 1 + t)) : 0.f;
    }
  }
#pragma unroll 4
  for (int i = 0; i < TT; ++i) {
    const int t = t0 + i;
    if (t >= L) break;
    float xv[V], o[V];
    Pack16<T>::load(xz + (size_t)(b * (size_t)L + t) * ld_xz + c, xv);
#pragma unroll
    for (int u = 0; u < V; ++u) {
      float acc = bc[u];
#pragma unroll
      for (int j = 0; j < K - 1; ++j) acc = fmaf(wk[u][j], win[u][j], acc);
      acc = fmaf(wk[u][K - 1], xv[u], acc);
#pragma unroll
      for (int j = 0; j < K - 2; ++j) win[u][j] = win[u][j + 1];
      win[u][K - 2] = xv[u];
      o[u] = silu_fast(acc);  // as the scan's conv phase
    }
    Pack16<T>::store(xc + (size_t)(b * (size_t)L + t) * ld_xc + c, o);
  }
}

// The vectorised conv with every input load of a thread issued before any arithmetic:
// a thread owns V channels (one 16-byte word per position) of P consecutive positions and
// first loads the P + K - 1 words it needs (the K - 1 halo re-read from L2 by the
// neighbouring position block) into registers, so each thread has P + K - 1 independent
// loads in flight instead of one per iteration -- the direct kernel above is bound by
// load latency, not bandwidth.  Same arithmetic, in the same order, as conv1d_silu_vec_kernel.
template <typename T, int K, int P>
__global__ void __launch_bounds__(128) conv1d_silu_batch_kernel(const T *__restrict__ xz, int ld_xz,
                                                                const T *__restrict__ w, const T *__restrict__ bias,
                                                                const T *__restrict__ hist, T *__restrict__ xc,
                                                                int ld_xc, int L, int Es, bool wvec) {
  MTP_PDL_WAIT();
  MTP_PDL_TRIGGER();
  constexpr int V = Pack16<T>::V;
  constexpr int W = P + K - 1;  // input words per thread
  static_assert(V * K * sizeof(T) == 64, "a group's taps are four 16-byte words");
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * V;
  const int t0 = blockIdx.y * P;
  const int b = blockIdx.z;
  if (c >= Es) return;
  // every input word first (positions t0 - K + 1 .. t0 + P - 1); out of range: zero, and
  // positions before the sequence start come from the history below
  uint4 raw[W];
  const T *xb = xz + (size_t)b * L * ld_xz + c;
#pragma unroll
  for (int i = 0; i < W; ++i) {
    const int t = t0 - (K - 1) + i;
    raw[i] = (t >= 0 && t < L) ? __ldg(reinterpret_cast<const uint4 *>(xb + (size_t)t * ld_xz)) : make_uint4(0, 0, 0, 0);
  }
  float wk[V][K], bc[V];
  if (wvec) {
    T tw[V * K], tb[V];
#pragma unroll
    for (int q = 0; q < 4; ++q) reinterpret_cast<uint4 *>(tw)[q] = __ldg(reinterpret_cast<const uint4 *>(w + (size_t)c * K) + q);
    if (bias) *reinterpret_cast<uint4 *>(tb) = __ldg(reinterpret_cast<const uint4 *>(bias + c));
#pragma unroll
    for (int u = 0; u < V; ++u) {
#pragma unroll
      for (int j = 0; j < K; ++j) wk[u][j] = ldf(&tw[u * K + j]);
      bc[u] = bias ? ldf(&tb[u]) : 0.f;
    }
  } else {
#pragma unroll
    for (int u = 0; u < V; ++u) {
#pragma unroll
      for (int j = 0; j < K; ++j) wk[u][j] = ldf(w + (size_t)(c + u) * K + j);
      bc[u] = bias ? ldf(bias + c + u) : 0.f;
    }
  }
  float win[V][K - 1];
#pragma unroll
  for (int j = 0; j < K - 1; ++j) {
    const int t = t0 - (K - 1) + j;
    if (t >= 0) {
      float v[V];
      Pack16<T>::load(reinterpret_cast<const T *>(&raw[j]), v);
#pragma unroll
      for (int u = 0; u < V; ++u) win[u][j] = v[u];
    } else {
#pragma unroll
      for (int u = 0; u < V; ++u) win[u][j] = hist ? ldf(hist + ((size_t)b * Es + c + u) * (K - 1) + (K - 1 + t)) : 0.f;
    }
  }
#pragma unroll
  for (int i = 0; i < P; ++i) {
    const int t = t0 + i;
    float xv[V], o[V];
    Pack16<T>::load(reinterpret_cast<const T *>(&raw[K - 1 + i]), xv);
#pragma unroll
    for (int u = 0; u < V; ++u) {
      float acc = bc[u];
#pragma unroll
      for (int j = 0; j < K - 1; ++j) acc = fmaf(wk[u][j], win[u][j], acc);
      acc = fmaf(wk[u][K - 1], xv[u], acc);
#pragma unroll
      for (int j = 0; j < K - 2; ++j) win[u][j] = win[u][j + 1];
      win[u][K - 2] = xv[u];
      o[u] = silu_fast(acc);
    }
    if (t < L) Pack16<T>::store(xc + ((size_t)b * L + t) * ld_xc + c, o);
  }
}

// The vectorised conv with its input staged in shared memory: every thread first issues one
// 16-byte cp.async per position of its column (TT + K - 1 of them, with the K - 1 halo),
// so a CTA has its whole input tile in flight at once without holding it in registers, then
// computes from shared memory.  Column of thread i at stage[p][i] (a warp reads 512
// contiguous bytes per position).  Same arithmetic as conv1d_silu_vec_kernel.
template <typename T, int K, int TT, int NTH>
__global__ void __launch_bounds__(NTH) conv1d_silu_smem_kernel(const T *__restrict__ xz, int ld_xz, const T *__restrict__ w,
                                                             const T *__restrict__ bias, const T *__restrict__ hist,
                                                             T *__restrict__ xc, int ld_xc, int L, int Es, bool wvec) {
  MTP_PDL_WAIT();
  MTP_PDL_TRIGGER();
  constexpr int V = Pack16<T>::V;
  extern __shared__ __align__(16) uint4 stage[];  // [TT + K - 1][NTH]
  const int c = (blockIdx.x * NTH + threadIdx.x) * V;
  const int t0 = blockIdx.y * TT;
  const int b = blockIdx.z;
  if (c >= Es) return;
  const int np = min(TT, L - t0) + (K - 1);
  for (int p = 0; p < np; ++p) {
    const int t = t0 - (K - 1) + p;
    uint4 *dst = &stage[p * NTH + threadIdx.x];
    if (t >= 0) {
      cp_async16(dst, xz + (size_t)(b * (size_t)L + t) * ld_xz + c);
    } else {  // before the sequence: the cache's conv history, or zeros
      T tv[V];
#pragma unroll
      for (int u = 0; u < V; ++u)
        tv[u] = hist ? hist[((size_t)b * Es + c + u) * (K - 1) + (K - 1 + t)] : (T)0.f;
      *dst = *reinterpret_cast<const uint4 *>(tv);
    }
  }
  cp_async_commit();
  float wk[V][K], bc[V];
  if (wvec) {
    T tw[V * K], tb[V];
#pragma unroll
    for (int q = 0; q < 4; ++q) reinterpret_cast<uint4 *>(tw)[q] = __ldg(reinterpret_cast<const uint4 *>(w + (size_t)c * K) + q);
    if (bias) *reinterpret_cast<uint4 *>(tb) = __ldg(reinterpret_cast<const uint4 *>(bias + c));
#pragma unroll
    for (int u = 0; u < V; ++u) {
#pragma unroll
      for (int j = 0; j < K; ++j) wk[u][j] = ldf(&tw[u * K + j]);
      bc[u] = bias ? ldf(&tb[u]) : 0.f;
    }
  } else {
#pragma unroll
    for (int u = 0; u < V; ++u) {
#pragma unroll
      for (int j = 0; j < K; ++j) wk[u][j] = ldf(w + (size_t)(c + u) * K + j);
      bc[u] = bias ? ldf(bias + c + u) : 0.f;
    }
  }
  cp_async_wait<0>();  // this thread's own column: no barrier needed
  float win[V][K - 1];
#pragma unroll
  for (int j = 0; j < K - 1; ++j) {
    float v[V];
    Pack16<T>::load(reinterpret_cast<const T *>(&stage[j * NTH + threadIdx.x]), v);
#pragma unroll
    for (int u = 0; u < V; ++u) win[u][j] = v[u];
  }
  const int tl = np - (K - 1);
#pragma unroll 4
  for (int i = 0; i < tl; ++i) {
    float xv[V], o[V];
    Pack16<T>::load(reinterpret_cast<const T *>(&stage[(i + K - 1) * NTH + threadIdx.x]), xv);
#pragma unroll
    for (int u = 0; u < V; ++u) {
      float acc = bc[u];
#pragma unroll
      for (int j = 0; j < K - 1; ++j) acc = fmaf(wk[u][j], win[u][j], acc);
      acc = fmaf(wk[u][K - 1], xv[u], acc);
#pragma unroll
      for (int j = 0; j < K - 2; ++j) win[u][j] = win[u][j + 1];
      win[u][K - 2] = xv[u];
      o[u] = silu_fast(acc);
    }
    Pack16<T>::store(xc + (size_t)(b * (size_t)L + t0 + i) * ld_xc + c, o);
  }
}

// ----------------------------------------------------------------- fused prefill scan
// CTA = 128 threads = (128 / TPC) channels of one sequence b; TPC threads share
// a channel, each holding N/TPC states in registers.  The sequence is walked in
// chunks of TL positions; raw x, z, dt and B|C of the next chunk are staged in
// shared memory by cp.async while the current one is processed.  Per chunk:
//   phase A  conv1d + SiLU of the TL positions (independent of the state: ILP)
//   phase B  the recurrence over the TL positions, storing y = (C.h + D.xc) * silu(z)
//            (a warp writes 32 consecutive channels of a position).
template <typename T, typename TD, int N, int TPC, int TL>
struct ScanSmem {
  static constexpr int CB = 128 / TPC;
  T x[2][TL][CB];
  T z[2][TL][CB];
  TD dt[2][TL][CB];
  float bc[2][TL][2 * N];
};




template <typename T, typename TD, int N, int TPC, int TL, int K>
__global__ void __launch_bounds__(128, (TPC == 1 ? 4 : 6)) scan_prefill_kernel(
    const T *__restrict__ xz, int ld_xz, const TD *__restrict__ dtp, int ld_dt, const float *__restrict__ bcp,
    int ld_bc, const T *__restrict__ A_log, const T *__restrict__ Dp, const T *__restrict__ conv_w,
    const T *__restrict__ conv_b, const T *conv_init, const float *ssm_init, T *__restrict__ y, int ld_y,
    T *conv_final, float *ssm_final, int L, int Es, bool vec16) {
  MTP_PDL_WAIT();
  MTP_PDL_TRIGGER();
  using S = ScanSmem<T, TD, N, TPC, TL>;
  constexpr int CB = S::CB;
  constexpr int NS = N / TPC;
  constexpr int NT = 128;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  S &sm = *reinterpret_cast<S *>(smem_raw);

  const int b = blockIdx.y;
  const int c0 = blockIdx.x * CB;
  const int cl = threadIdx.x / TPC;
  const int sub = threadIdx.x % TPC;
  const int c = c0 + cl;
  const bool live = c < Es;
  const int ncb = min(CB, Es - c0);
  const size_t row0 = (size_t)b * L;

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

  auto load_chunk = [&](int k, int buf) {
    const int t0 = k * TL;
    const int tl = min(TL, L - t0);
    if (vec16) {  // full channel blocks, 16-byte aligned rows
      constexpr int XW = CB * (int)sizeof(T) / 16, DW = CB * (int)sizeof(TD) / 16, BW = 2 * N * 4 / 16;
      constexpr int DE = 16 / (int)sizeof(TD);  // dt elements per 16-byte granule
      for (int i = threadIdx.x; i < tl * XW; i += NT) {
        const int tt = i / XW, w = i % XW;
        const T *src = xz + (row0 + t0 + tt) * ld_xz + c0;
        cp_async16(reinterpret_cast<char *>(&sm.x[buf][tt][0]) + 16 * w, reinterpret_cast<const char *>(src) + 16 * w);
        cp_async16(reinterpret_cast<char *>(&sm.z[buf][tt][0]) + 16 * w,
                   reinterpret_cast<const char *>(src + Es) + 16 * w);
      }
      for (int i = threadIdx.x; i < tl * DW; i += NT) {
        const int tt = i / DW, w = i % DW;
        cp_async16(&sm.dt[buf][tt][DE * w], dtp + (row0 + t0 + tt) * ld_dt + c0 + DE * w);
      }
      for (int i = threadIdx.x; i < tl * BW; i += NT) {
        const int tt = i / BW, w = i % BW;
        cp_async16(&sm.bc[buf][tt][4 * w], bcp + (row0 + t0 + tt) * ld_bc + 4 * w);
      }
    } else {  // 4-byte granules, partial channel blocks
      constexpr int EPW = 4 / sizeof(T);
      const int wpr = (ncb + EPW - 1) / EPW;
      for (int i = threadIdx.x; i < tl * wpr; i += NT) {
        const int tt = i / wpr, wi = i % wpr;
        cp_async4(&sm.x[buf][tt][wi * EPW], xz + (row0 + t0 + tt) * ld_xz + c0 + wi * EPW);
        cp_async4(&sm.z[buf][tt][wi * EPW], xz + (row0 + t0 + tt) * ld_xz + Es + c0 + wi * EPW);
      }
      constexpr int DPW = 4 / sizeof(TD);
      const int dpr = (ncb + DPW - 1) / DPW;
      for (int i = threadIdx.x; i < tl * dpr; i += NT) {
        const int tt = i / dpr, wi = i % dpr;
        cp_async4(&sm.dt[buf][tt][wi * DPW], dtp + (row0 + t0 + tt) * ld_dt + c0 + wi * DPW);
      }
      for (int i = threadIdx.x; i < tl * 2 * N; i += NT) {
        const int tt = i / (2 * N), j = i % (2 * N);
        cp_async4(&sm.bc[buf][tt][j], bcp + (row0 + t0 + tt) * ld_bc + j);
      }
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
    // phase A: conv + SiLU for the chunk (every lane runs it; lanes past the last
    // channel read in-bounds shared memory and store nothing)
    float xcs[TL], dts[TL];
#pragma unroll
    for (int tt = 0; tt < TL; ++tt) {
      if (tt < tl) {
        const float xv = ldf(&sm.x[buf][tt][cl]);
        float acc = cbias;
#pragma unroll
        for (int j = 0; j < K - 1; ++j) acc = fmaf(wk[j], win[j], acc);
        acc = fmaf(wk[K - 1], xv, acc);
#pragma unroll
        for (int j = 0; j < K - 2; ++j) win[j] = win[j + 1];
        win[K - 2] = xv;
        xcs[tt] = silu_fast(acc);
        dts[tt] = ldf(&sm.dt[buf][tt][cl]);
      }
    }
    // phase B: recurrence
#pragma unroll
    for (int tt = 0; tt < TL; ++tt) {
      if (tt < tl) {
        const float dt = dts[tt];
        const float dtx = dt * xcs[tt];
        const float4 *bv = reinterpret_cast<const float4 *>(&sm.bc[buf][tt][sub * NS]);
        const float4 *cv = reinterpret_cast<const float4 *>(&sm.bc[buf][tt][N + sub * NS]);
        float ya[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int q = 0; q < NS / 4; ++q) {
          const float4 B4 = bv[q], C4 = cv[q];
          const float Bs[4] = {B4.x, B4.y, B4.z, B4.w}, Cs[4] = {C4.x, C4.y, C4.z, C4.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int i = 4 * q + u;
            const float dA = ex2_hw(dt * A2[i]);
            h[i] = fmaf(dA, h[i], Bs[u] * dtx);
            ya[u] = fmaf(Cs[u], h[i], ya[u]);
          }
        }
        float yv = (ya[0] + ya[1]) + (ya[2] + ya[3]);
#pragma unroll
        for (int o = 1; o < TPC; o <<= 1) yv += __shfl_xor_sync(0xffffffffu, yv, o);
        if (sub == 0 && live)
          stf(y + (row0 + t0 + tt) * ld_y + c, fmaf(Dv, xcs[tt], yv) * silu_fast(ldf(&sm.z[buf][tt][cl])));
      }
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

// ----------------------------------------------------------------- scan over the conv output
// The recurrence of the fused prefill above, fed with xc = SiLU(conv1d(x)) as written by
// conv1d_silu_vec_kernel for x_proj (so the scan spends no SFU work on the conv), with
// the SFU load cut further:
//   * the state update runs on packed fp32 pairs (fma.rn.f32x2 / mul.rn.f32x2, sm_100a);
//   * NPP of the thread's N/(2 TPC) state pairs take exp2 on the FP32 pipe
//     (exp2_poly2 below) instead of the MUFU unit, which stays the limit otherwise;
//   * bf16 models gate with silu(z) = h + h tanh(h), h = z/2 (one tanh.approx,
//     |error| <= 2.5e-4 of |z|, below a bf16 step); fp32 models keep z / (1 + e^-z).
// TPC threads share a channel; for TPC > 1 the gate of position tt is computed and
// y stored by lane tt % TPC of the channel, spreading that work over the lanes.

// 2^x, x <= 0, on the FP32 pipe, for a pair of values.  Range reduction in the style of
// Cody and Waite: j = rint(x) through the 1.5 * 2^23 rounding constant (the sum's low
// mantissa bits hold j), f = x - j in [-1/2, 1/2]; 2^f by a degree-5 polynomial fitted for
// minimum relative error on [-1/2, 1/2] with the Remez exchange algorithm
// (csrc/fit_exp2_poly.py prints these coefficients); 2^j is added into the exponent field.
// Relative error <= 2.4e-7 (fp32 Horner included) for x in [-125, 0]; x < -125 gives
// 2^-125 (the ex2.approx.ftz result there is 0; both are negligible as a state decay).
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float RND = 12582912.0f;  // 1.5 * 2^23
  constexpr float P0 = 1.0000001192092896f, P1 = 0.6931469440460205f, P2 = 0.24022120237350464f,
                  P3 = 0.05550713092088699f, P4 = 0.009675540961325169f, P5 = 0.0013276472454890609f;
  x.x = fmaxf(x.x, -125.0f);
  x.y = fmaxf(x.y, -125.0f);
  const float2 t = __fadd2_rn(x, make_float2(RND, RND));
  const float2 nj = __ffma2_rn(t, make_float2(-1.0f, -1.0f), make_float2(RND, RND));  // -rint(x), exact
  const float2 f = __fadd2_rn(x, nj);
  float2 p = __ffma2_rn(make_float2(P5, P5), f, make_float2(P4, P4));
  p = __ffma2_rn(p, f, make_float2(P3, P3));
  p = __ffma2_rn(p, f, make_float2(P2, P2));
  p = __ffma2_rn(p, f, make_float2(P1, P1));
  p = __ffma2_rn(p, f, make_float2(P0, P0));
  // the rounded sum's bits are 0x4B400000 + j; shifted by 23 only j << 23 survives (mod 2^32)
  return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}

__device__ __forceinline__ float tanh_hw(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T> __device__ __forceinline__ float gate_silu(float z);
template <> __device__ __forceinline__ float gate_silu<__nv_bfloat16>(float z) {
  const float h = 0.5f * z;
  return fmaf(h, tanh_hw(h), h);
}
template <> __device__ __forceinline__ float gate_silu<float>(float z) { return silu_fast(z); }

__global__ void exp2_fma_kernel(const float *__restrict__ x, float *__restrict__ out, int n) {
  MTP_PDL_WAIT();
  MTP_PDL_TRIGGER();
  const int i = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (i >= n) return;
  const float2 v = exp2_poly2(make_float2(x[i], i + 1 < n ? x[i + 1] : 0.f));
  out[i] = v.x;
  if (i + 1 < n) out[i + 1] = v.y;
}

template <typename T, typename TD, int N, int TPC, int TL>
struct ScanXcSmem {
  static constexpr int CB = 128 / TPC;
  T xc[2][TL][CB];
  T z[2][TL][CB];
  TD dt[2][TL][CB];
  float bc[2][TL][2 * N];
};

// Sequence chunks (few independent recurrences per SM, e.g. 640 channels x 8 sequences):
// blockIdx.z = chunk k covers positions [k Lc, min(L, (k+1) Lc)) of every sequence.  ST = true
// is the state pass: the chunk's end state from a zero state, E_k, and its sum of dt, S_k,
// into slot k of chunk_io [B][NC][Es][N + 1] (no outputs); its chunk-0 CTAs also copy the
// initial state into slot NC - 1 (the last chunk needs no end state), because the output
// pass may overwrite ssm_init in place (ssm_final aliasing it) while other chunks still need
// it.  ST = false starts chunk k from h = exp2(A2 S_{k-1}) (... (exp2(A2 S_0) h_init + E_0) ...)
// + E_{k-1} and writes y for the chunk, the last chunk also the final state and conv history.
// (exp2(A2 S) is the product of the chunk's per-position decays up to rounding.)  Unchunked:
// NC = 1, Lc = L, h_init read from ssm_init.
template <typename T, typename TD, int N, int TPC, int TL, int K, int NPP, int MINB, bool ST>
__global__ void __launch_bounds__(128, MINB) scan_xc_kernel(
    const T *__restrict__ xc, int ld_xc, const T *__restrict__ xz, int ld_xz, const TD *__restrict__ dtp, int ld_dt,
    const float *__restrict__ bcp, int ld_bc, const T *__restrict__ A_log, const T *__restrict__ Dp,
    const T *conv_init, const float *ssm_init, T *__restrict__ y, int ld_y, T *conv_final, float *ssm_final,
    int Lseq, int Es, bool vec16, int Lc, int NC, float *chunk_io) {
  MTP_PDL_WAIT();
  MTP_PDL_TRIGGER();
  using S = ScanXcSmem<T, TD, N, TPC, TL>;
  constexpr int CB = S::CB;
  constexpr int NS = N / TPC;  // states per thread
  constexpr int NP = NS / 2;   // state pairs per thread
  static_assert(NS % 4 == 0 && NPP <= NP, "states per thread: a multiple of 4");
  constexpr int NT = 128;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  S &sm = *reinterpret_cast<S *>(smem_raw);

  const int b = blockIdx.y;
  const int kz = blockIdx.z;
  const int c0 = blockIdx.x * CB;
  const int cl = threadIdx.x / TPC;
  const int sub = threadIdx.x % TPC;
  const int c = c0 + cl;
  const bool live = c < Es;
  const int ncb = min(CB, Es - c0);
  const int tb = kz * Lc;
  const int L = min(Lc, Lseq - tb);  // positions of this chunk
  const size_t row0 = (size_t)b * Lseq + tb;

  float2 A2[NP], h[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int n = sub * NS + 2 * i;
    A2[i].x = live ? -expf(ldf(A_log + (size_t)c * N + n)) * kLog2e : 0.f;
    A2[i].y = live ? -expf(ldf(A_log + (size_t)c * N + n + 1)) * kLog2e : 0.f;
    h[i] = make_float2(0.f, 0.f);
    if (live && ssm_init && (ST ? kz == 0 : NC == 1)) {  // the state pass copies it (below)
      h[i].x = ssm_init[((size_t)b * Es + c) * N + n];
      h[i].y = ssm_init[((size_t)b * Es + c) * N + n + 1];
    }
    if (!ST && NC > 1 && live && ssm_init) {  // the copy taken by the state pass
      const float *ini = chunk_io + (((size_t)b * NC + NC - 1) * Es + c) * (N + 1);
      h[i] = make_float2(ini[n], ini[n + 1]);
    }
  }
  if (ST && kz == 0 && live && ssm_init) {
    float *ini = chunk_io + (((size_t)b * NC + NC - 1) * Es + c) * (N + 1);
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      ini[sub * NS + 2 * i] = h[i].x;
      ini[sub * NS + 2 * i + 1] = h[i].y;
      h[i] = make_float2(0.f, 0.f);  // the end state of chunk 0 is taken from zero too
    }
  }
  if (!ST && live) {  // carry the state through the earlier chunks
    for (int jz = 0; jz < kz; ++jz) {
      const float *io = chunk_io + (((size_t)b * NC + jz) * Es + c) * (N + 1);
      const float sdt = io[N];
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        const int n = sub * NS + 2 * i;
        const float2 dec = make_float2(ex2_hw(A2[i].x * sdt), ex2_hw(A2[i].y * sdt));
        h[i] = __ffma2_rn(dec, h[i], make_float2(io[n], io[n + 1]));
      }
    }
  }
  float ssum = 0.f;  // state pass: sum of dt over the chunk
  const float Dv = live ? ldf(Dp + c) : 0.f;

  auto load_chunk = [&](int k, int buf) {
    const int t0 = k * TL;
    const int tl = min(TL, L - t0);
    if (vec16) {  // full channel blocks, 16-byte aligned rows
      constexpr int XW = CB * (int)sizeof(T) / 16, DW = CB * (int)sizeof(TD) / 16, BW = 2 * N * 4 / 16;
      constexpr int DE = 16 / (int)sizeof(TD);
      for (int i = threadIdx.x; i < tl * XW; i += NT) {
        const int tt = i / XW, w = i % XW;
        cp_async16(reinterpret_cast<char *>(&sm.xc[buf][tt][0]) + 16 * w,
                   reinterpret_cast<const char *>(xc + (row0 + t0 + tt) * ld_xc + c0) + 16 * w);
        cp_async16(reinterpret_cast<char *>(&sm.z[buf][tt][0]) + 16 * w,
                   reinterpret_cast<const char *>(xz + (row0 + t0 + tt) * ld_xz + Es + c0) + 16 * w);
      }
      for (int i = threadIdx.x; i < tl * DW; i += NT) {
        const int tt = i / DW, w = i % DW;
        cp_async16(&sm.dt[buf][tt][DE * w], dtp + (row0 + t0 + tt) * ld_dt + c0 + DE * w);
      }
      for (int i = threadIdx.x; i < tl * BW; i += NT) {
        const int tt = i / BW, w = i % BW;
        cp_async16(&sm.bc[buf][tt][4 * w], bcp + (row0 + t0 + tt) * ld_bc + 4 * w);
      }
    } else {  // 4-byte granules, partial channel blocks
      constexpr int EPW = 4 / sizeof(T);
      const int wpr = (ncb + EPW - 1) / EPW;
      for (int i = threadIdx.x; i < tl * wpr; i += NT) {
        const int tt = i / wpr, wi = i % wpr;
        cp_async4(&sm.xc[buf][tt][wi * EPW], xc + (row0 + t0 + tt) * ld_xc + c0 + wi * EPW);
        cp_async4(&sm.z[buf][tt][wi * EPW], xz + (row0 + t0 + tt) * ld_xz + Es + c0 + wi * EPW);
      }
      constexpr int DPW = 4 / sizeof(TD);
      const int dpr = (ncb + DPW - 1) / DPW;
      for (int i = threadIdx.x; i < tl * dpr; i += NT) {
        const int tt = i / dpr, wi = i % dpr;
        cp_async4(&sm.dt[buf][tt][wi * DPW], dtp + (row0 + t0 + tt) * ld_dt + c0 + wi * DPW);
      }
      for (int i = threadIdx.x; i < tl * 2 * N; i += NT) {
        const int tt = i / (2 * N), j = i % (2 * N);
        cp_async4(&sm.bc[buf][tt][j], bcp + (row0 + t0 + tt) * ld_bc + j);
      }
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
    // TPC > 1: gates of the positions this lane stores, tt = sub + TPC * i, computed up
    // front (one lane per position); TPC == 1 gates each position where it is stored
    constexpr int NG = TPC == 1 ? 1 : TL / TPC;
    float gt[NG];
    if constexpr (TPC > 1 && !ST) {
#pragma unroll
      for (int i = 0; i < NG; ++i) {
        const int tt = sub + TPC * i;
        gt[i] = tt < tl ? gate_silu<T>(ldf(&sm.z[buf][tt][cl])) : 0.f;
      }
    }
    T *ychunk = y + (row0 + t0) * ld_y + c;
    auto token = [&](const int tt) {
      const float xv = ldf(&sm.xc[buf][tt][cl]);
      const float dt = ldf(&sm.dt[buf][tt][cl]);
      if constexpr (ST) {  // state pass: the recurrence and the sum of dt only
        const float2 dt2 = make_float2(dt, dt);
        const float2 dtx2 = make_float2(dt * xv, dt * xv);
        const float4 *bv = reinterpret_cast<const float4 *>(&sm.bc[buf][tt][sub * NS]);
        ssum += dt;
#pragma unroll
        for (int q = 0; q < NS / 4; ++q) {
          const float4 B4 = bv[q];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int i = 2 * q + u;
            const float2 Bp = u ? make_float2(B4.z, B4.w) : make_float2(B4.x, B4.y);
            const float2 arg = __fmul2_rn(dt2, A2[i]);
            const float2 dA = make_float2(ex2_hw(arg.x), ex2_hw(arg.y));
            h[i] = __ffma2_rn(dA, h[i], __fmul2_rn(Bp, dtx2));
          }
        }
        return;
      }
      const float2 dt2 = make_float2(dt, dt);
      const float dtx = dt * xv;
      const float2 dtx2 = make_float2(dtx, dtx);
      const float4 *bv = reinterpret_cast<const float4 *>(&sm.bc[buf][tt][sub * NS]);
      const float4 *cv = reinterpret_cast<const float4 *>(&sm.bc[buf][tt][N + sub * NS]);
      float2 ya = make_float2(0.f, 0.f), yb = make_float2(0.f, 0.f);
#pragma unroll
      for (int q = 0; q < NS / 4; ++q) {
        const float4 B4 = bv[q], C4 = cv[q];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int i = 2 * q + u;
          const float2 Bp = u ? make_float2(B4.z, B4.w) : make_float2(B4.x, B4.y);
          const float2 Cp = u ? make_float2(C4.z, C4.w) : make_float2(C4.x, C4.y);
          const float2 arg = __fmul2_rn(dt2, A2[i]);
          float2 dA;
          if (i < NPP) {
            dA = exp2_poly2(arg);
          } else {
            dA.x = ex2_hw(arg.x);
            dA.y = ex2_hw(arg.y);
          }
          h[i] = __ffma2_rn(dA, h[i], __fmul2_rn(Bp, dtx2));
          if (u) yb = __ffma2_rn(Cp, h[i], yb);
          else ya = __ffma2_rn(Cp, h[i], ya);
        }
      }
      const float2 ys = __fadd2_rn(ya, yb);
      float yv = ys.x + ys.y;
#pragma unroll
      for (int o = 1; o < TPC; o <<= 1) yv += __shfl_xor_sync(0xffffffffu, yv, o);
      if constexpr (TPC == 1) {
        if (live) stf(ychunk + (size_t)tt * ld_y, fmaf(Dv, xv, yv) * gate_silu<T>(ldf(&sm.z[buf][tt][cl])));
      } else {
        if (sub == tt % TPC && live) stf(ychunk + (size_t)tt * ld_y, fmaf(Dv, xv, yv) * gt[tt / TPC]);
      }
    };
    // (a guard-free copy of this loop for full chunks measured slower: the interleaving it
    // allows spills registers)
#pragma unroll
    for (int tt = 0; tt < TL; ++tt)
      if (tt < tl) token(tt);
    // buffer `buf` is refilled by the next iteration's prefetch only after this barrier
    __syncthreads();
  }
  if (ST) {  // chunk end state from zero and its sum of dt
    if (live) {
      float *io = chunk_io + (((size_t)b * NC + kz) * Es + c) * (N + 1);
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        io[sub * NS + 2 * i] = h[i].x;
        io[sub * NS + 2 * i + 1] = h[i].y;
      }
      if (sub == 0) io[N] = ssum;
    }
    return;
  }
  if (live && kz == NC - 1) {
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      ssm_final[((size_t)b * Es + c) * N + sub * NS + 2 * i] = h[i].x;
      ssm_final[((size_t)b * Es + c) * N + sub * NS + 2 * i + 1] = h[i].y;
    }
    if (sub == 0) {
      // conv history for the next prefill: the last K-1 inputs of [conv_init | x] of the
      // whole sequence (all read before any write: conv_final may alias conv_init)
      float hv[K - 1];
#pragma unroll
      for (int j = 0; j < K - 1; ++j) {
        const int t = Lseq - (K - 1) + j;
        hv[j] = t >= 0 ? ldf(xz + ((size_t)b * Lseq + t) * ld_xz + c)
                       : (conv_init ? ldf(conv_init + ((size_t)b * Es + c) * (K - 1) + (K - 1 + t)) : 0.f);
      }
#pragma unroll
      for (int j = 0; j < K - 1; ++j) stf(conv_final + ((size_t)b * Es + c) * (K - 1) + j, hv[j]);
    }
  }
}

// ----------------------------------------------------------------- fused dt_proj + scan (bf16)
// The scan above with dt_proj (+ bias + softplus) computed inside the kernel on
// the tensor cores: per chunk of TL positions, D[128 channels x TL positions] =
// W_dt[c0:c0+128, :R] . dt_low[rows, :R]^T as tcgen05.mma (M=128, N=TL, K=16 per
// instruction), operands staged by TMA with 128-byte swizzle, fp32 accumulators
// double-buffered in TMEM.  TMEM lane i holds channel c0+i, so tcgen05.ld 32x32b
// gives each thread its own channel's dt for the chunk.  Thread 0 issues the TMA
// loads (two chunks ahead) and the MMA of chunk k+1 while chunk k is scanned.
// Every mbarrier wait is bounded; a timeout sets a device status word and all
// threads leave the chunk loop together.
template <int TL, int KA>
struct FusedSmem {
  uint8_t w[KA][128 * 128];     // W_dt tile: 128 rows x 64 columns per atom (1024-aligned)
  uint8_t dl[2][KA][TL * 128];  // dt_low tiles of two chunks
  __nv_bfloat16 x[2][TL][128];
  __nv_bfloat16 z[2][TL][128];
  float bc[2][TL][32];
  uint64_t bar_w, bar_dl[2], bar_mma[2];
  uint32_t tmem;
  int abort;
};

template <int TL, int KA, int K>
__global__ void __launch_bounds__(128, 4) scan_fused_kernel(
    const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_dl,
    const __nv_bfloat16 *__restrict__ xz, int ld_xz, const __nv_bfloat16 *__restrict__ b_dt,
    const float *__restrict__ bcp, int ld_bc, const __nv_bfloat16 *__restrict__ A_log,
    const __nv_bfloat16 *__restrict__ Dp, const __nv_bfloat16 *__restrict__ conv_w,
    const __nv_bfloat16 *__restrict__ conv_b, const __nv_bfloat16 *conv_init, const float *ssm_init,
    __nv_bfloat16 *__restrict__ y, int ld_y, __nv_bfloat16 *conv_final, float *ssm_final, int L, int Es, int *err,
    unsigned long long timeout_ns) {
  using namespace tc;
  constexpr int N = 16, CB = 128, NT = 128;
  using S = FusedSmem<TL, KA>;
  extern __shared__ __align__(1024) unsigned char smem_dyn[];
  const uint32_t raw = smem_u32(smem_dyn);
  const uint32_t base = (raw + 1023u) & ~1023u;
  S &sm = *reinterpret_cast<S *>(smem_dyn + (base - raw));
  const int tid = threadIdx.x, warp = tid >> 5;
  const int b = blockIdx.y, c0 = blockIdx.x * CB, c = c0 + tid;
  const size_t row0 = (size_t)b * L;
  const int nchunks = (L + TL - 1) / TL;
  constexpr uint32_t W_BYTES = KA * 128 * 128, DL_BYTES = KA * TL * 128;
  const uint32_t idesc = idesc_bf16(128, TL);
  volatile int *abort = &sm.abort;

  if (tid == 0) {
    mbar_init(smem_u32(&sm.bar_w), 1);
    for (int j = 0; j < 2; ++j) {
      mbar_init(smem_u32(&sm.bar_dl[j]), 1);
      mbar_init(smem_u32(&sm.bar_mma[j]), 1);
    }
    sm.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm.tmem)), "r"(32));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  MTP_PDL_WAIT();  // barrier init and TMEM allocation above overlap the previous kernel
  MTP_PDL_TRIGGER();
  const uint32_t tmem = sm.tmem;

  auto issue_dl = [&](int chunk, int bufi) {  // thread 0
    mbar_expect_tx(smem_u32(&sm.bar_dl[bufi]), DL_BYTES);
    for (int a = 0; a < KA; ++a)
      tma_load_2d(smem_u32(&sm.dl[bufi][a][0]), &tm_dl, smem_u32(&sm.bar_dl[bufi]), 64 * a, (int)(row0 + chunk * TL));
  };
  auto issue_mma = [&](int bufi) {  // thread 0, after the chunk's dt_low landed
    const uint32_t d = tmem + (uint32_t)(bufi * TL);
    for (int a = 0; a < KA; ++a) {
      const uint64_t ad = sw128_desc(smem_u32(&sm.w[a][0])), bd = sw128_desc(smem_u32(&sm.dl[bufi][a][0]));
#pragma unroll
      for (int k = 0; k < 4; ++k) umma_bf16(d, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc, (a | k) != 0);
    }
    umma_commit(smem_u32(&sm.bar_mma[bufi]));
  };

  if (tid == 0) {
    mbar_expect_tx(smem_u32(&sm.bar_w), W_BYTES);
    for (int a = 0; a < KA; ++a) tma_load_2d(smem_u32(&sm.w[a][0]), &tm_w, smem_u32(&sm.bar_w), 64 * a, c0);
    issue_dl(0, 0);
    if (nchunks > 1) issue_dl(1, 1);
    if (mbar_wait(smem_u32(&sm.bar_w), 0, abort, timeout_ns) && mbar_wait(smem_u32(&sm.bar_dl[0]), 0, abort, timeout_ns)) {
      tc_fence_after();
      issue_mma(0);
    } else {
      *abort = 1;
    }
  }

  // per-thread constants
  float A2[N], h[N], wk[K], win[K - 1];
#pragma unroll
  for (int i = 0; i < N; ++i) {
    A2[i] = -expf(__bfloat162float(A_log[(size_t)c * N + i])) * kLog2e;
    h[i] = ssm_init ? ssm_init[((size_t)b * Es + c) * N + i] : 0.f;
  }
#pragma unroll
  for (int j = 0; j < K; ++j) wk[j] = __bfloat162float(conv_w[(size_t)c * K + j]);
#pragma unroll
  for (int j = 0; j < K - 1; ++j) win[j] = conv_init ? __bfloat162float(conv_init[((size_t)b * Es + c) * (K - 1) + j]) : 0.f;
  const float Dv = __bfloat162float(Dp[c]);
  const float cbias = conv_b ? __bfloat162float(conv_b[c]) : 0.f;
  const float bdt = __bfloat162float(b_dt[c]);

  auto load_chunk = [&](int k, int bufi) {
    const int t0 = k * TL;
    const int tl = min(TL, L - t0);
    constexpr int XW = CB * 2 / 16, BW = 2 * N * 4 / 16;
    for (int i = tid; i < tl * XW; i += NT) {
      const int tt = i / XW, w = i % XW;
      const __nv_bfloat16 *src = xz + (row0 + t0 + tt) * ld_xz + c0;
      cp_async16(reinterpret_cast<char *>(&sm.x[bufi][tt][0]) + 16 * w, reinterpret_cast<const char *>(src) + 16 * w);
      cp_async16(reinterpret_cast<char *>(&sm.z[bufi][tt][0]) + 16 * w, reinterpret_cast<const char *>(src + Es) + 16 * w);
    }
    for (int i = tid; i < tl * BW; i += NT) {
      const int tt = i / BW, w = i % BW;
      cp_async16(&sm.bc[bufi][tt][4 * w], bcp + (row0 + t0 + tt) * ld_bc + 4 * w);
    }
    cp_async_commit();
  };

  load_chunk(0, 0);
  for (int k = 0; k < nchunks; ++k) {
    const int buf = k & 1;
    if (k + 1 < nchunks) {
      load_chunk(k + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    // dt of this chunk from TMEM
    if (!mbar_wait(smem_u32(&sm.bar_mma[buf]), (uint32_t)((k >> 1) & 1), abort, timeout_ns)) *abort = 1;
    __syncthreads();
    if (*abort) break;
    tc_fence_after();
    float dts[TL];
    tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(buf * TL), dts);
    if (tid == 0) {
      // the MMA of chunk k read dl[buf]: refill it two chunks ahead, then start chunk k+1's MMA
      if (k + 2 < nchunks) issue_dl(k + 2, buf);
      if (k + 1 < nchunks) {
        if (mbar_wait(smem_u32(&sm.bar_dl[buf ^ 1]), (uint32_t)(((k + 1) >> 1) & 1), abort, timeout_ns)) {
          tc_fence_after();
          issue_mma(buf ^ 1);
        } else {
          *abort = 1;
        }
      }
    }
#pragma unroll
    for (int tt = 0; tt < TL; ++tt) dts[tt] = softplus_fast(dts[tt] + bdt);
    const int t0 = k * TL;
    const int tl = min(TL, L - t0);
    float xcs[TL];
#pragma unroll
    for (int tt = 0; tt < TL; ++tt) {
      if (tt < tl) {
        const float xv = __bfloat162float(sm.x[buf][tt][tid]);
        float acc = cbias;
#pragma unroll
        for (int j = 0; j < K - 1; ++j) acc = fmaf(wk[j], win[j], acc);
        acc = fmaf(wk[K - 1], xv, acc);
#pragma unroll
        for (int j = 0; j < K - 2; ++j) win[j] = win[j + 1];
        win[K - 2] = xv;
        xcs[tt] = silu_fast(acc);
      }
    }
#pragma unroll
    for (int tt = 0; tt < TL; ++tt) {
      if (tt < tl) {
        const float dt = dts[tt];
        const float dtx = dt * xcs[tt];
        const float4 *bv = reinterpret_cast<const float4 *>(&sm.bc[buf][tt][0]);
        const float4 *cv = reinterpret_cast<const float4 *>(&sm.bc[buf][tt][N]);
        float ya[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int q = 0; q < N / 4; ++q) {
          const float4 B4 = bv[q], C4 = cv[q];
          const float Bs[4] = {B4.x, B4.y, B4.z, B4.w}, Cs[4] = {C4.x, C4.y, C4.z, C4.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int i = 4 * q + u;
            const float dA = ex2_hw(dt * A2[i]);
            h[i] = fmaf(dA, h[i], Bs[u] * dtx);
            ya[u] = fmaf(Cs[u], h[i], ya[u]);
          }
        }
        const float yv = fmaf(Dv, xcs[tt], (ya[0] + ya[1]) + (ya[2] + ya[3]));
        y[(row0 + t0 + tt) * ld_y + c] = __float2bfloat16_rn(yv * silu_fast(__bfloat162float(sm.z[buf][tt][tid])));
      }
    }
    tc_fence_before();
    __syncthreads();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (*abort) {
    if (tid == 0) {
      atomicExch(err, MTP_ERR_TIMEOUT);
      const unsigned long long t0 = globaltimer_ns();  // let copies / MMAs in flight finish
      while (globaltimer_ns() - t0 < 1000000ull) {}
    }
    __syncthreads();
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) ssm_final[((size_t)b * Es + c) * N + i] = h[i];
#pragma unroll
    for (int j = 0; j < K - 1; ++j) conv_final[((size_t)b * Es + c) * (K - 1) + j] = __float2bfloat16_rn(win[j]);
  }
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(32));
}

static int *scan_err_word() {
  static int *w = nullptr;
  if (!w) {
    if (cudaMalloc(&w, sizeof(int)) != cudaSuccess) return nullptr;
    cudaMemset(w, 0, sizeof(int));
  }
  return w;
}

template <int KA>
static int launch_scan_fused(const void *xz, int ld_xz, const void *dt_low, int ld_dl, const void *W_dt,
                             const void *b_dt, const float *bc, int ld_bc, const void *A_log, const void *Dp,
                             const void *conv_w, const void *conv_b, const void *conv_init, const float *ssm_init,
                             void *y, int ld_y, void *conv_final, float *ssm_final, int B, int L, int Es, int R,
                             cudaStream_t s) {
  constexpr int TL = 16, K = 4;
  using S = FusedSmem<TL, KA>;
  const int smem = (int)sizeof(S) + 1024;
  auto kern = scan_fused_kernel<TL, KA, K>;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return check_launch("scan_fused attr");
    attr_set = true;
  }
  CUtensorMap tw, td;
  int rc = tc::make_tmap(&tw, W_dt, Es, R, R, 128);
  if (rc) return rc;
  rc = tc::make_tmap(&td, dt_low, B * L, R, ld_dl, TL);
  if (rc) return rc;
  int *err = scan_err_word();
  if (!err) return fail(MTP_ERR_CUDA, "could not allocate the scan status word");
  dim3 grid(Es / 128, B);
  launch_pdl(kern, dim3(grid), dim3(128), smem, s, tw, td, (const __nv_bfloat16 *)xz, ld_xz, (const __nv_bfloat16 *)b_dt, bc, ld_bc,
                               (const __nv_bfloat16 *)A_log, (const __nv_bfloat16 *)Dp, (const __nv_bfloat16 *)conv_w,
                               (const __nv_bfloat16 *)conv_b, (const __nv_bfloat16 *)conv_init, ssm_init,
                               (__nv_bfloat16 *)y, ld_y, (__nv_bfloat16 *)conv_final, ssm_final, L, Es, err,
                               2000000000ull);
  return check_launch("scan_fused");
}

// ----------------------------------------------------------------- single-token step
// CTA = 32 channels x BB sequences, one thread per (sequence, channel) holding
// all N states.  The block's dt_proj rows are staged transposed in shared memory
// ([R][33]: conflict-free across the 32 channels of a warp) with the BB dt_low
// vectors and A * log2(e); each thread then does its dt_proj dot product,
// softplus, the conv over [history | x] with the history shift, the state
// update (float4), C.h, the D skip and the SiLU(z) gate, all in place.
template <typename T, int N, int K>
__global__ void __launch_bounds__(256) step_kernel(const T *__restrict__ xz, int ld_xz, const T *__restrict__ dt_low,
                                                   int ld_dl, const T *__restrict__ W_dt, const T *__restrict__ b_dt,
                                                   const float *__restrict__ bcp, int ld_bc, const T *__restrict__ A_log,
                                                   const T *__restrict__ Dp, const T *__restrict__ conv_w,
                                                   const T *__restrict__ conv_b, T *conv_state, float *ssm_state,
                                                   T *__restrict__ y, int ld_y, int B, int Es, int R, int BB) {
  MTP_PDL_WAIT();
  MTP_PDL_TRIGGER();
  constexpr int CB = 32;
  extern __shared__ __align__(16) float ssm_sm[];
  // staging uses all 256 threads; the first 32 x BB threads then own one (sequence, channel) each
  float *wt = ssm_sm;                   // [R][CB + 1]
  float *dls = wt + R * (CB + 1);       // [BB][R]
  float *a2s = dls + BB * R;            // [CB][N]
  const int c0 = blockIdx.x * CB, b0 = blockIdx.y * BB;
  const int ncb = min(CB, Es - c0), nbb = min(BB, B - b0);
  for (int i = threadIdx.x; i < ncb * R; i += blockDim.x) {
    const int cc = i / R, r = i % R;
    wt[r * (CB + 1) + cc] = ldf(W_dt + (size_t)(c0 + cc) * R + r);
  }
  for (int i = threadIdx.x; i < nbb * R; i += blockDim.x) {
    const int bb = i / R, r = i % R;
    dls[bb * R + r] = ldf(dt_low + (size_t)(b0 + bb) * ld_dl + r);
  }
  for (int i = threadIdx.x; i < ncb * N; i += blockDim.x)
    a2s[i] = -expf(ldf(A_log + (size_t)c0 * N + i)) * kLog2e;
  __syncthreads();
  const int bl = threadIdx.x / CB, cl = threadIdx.x % CB;
  const int b = b0 + bl, c = c0 + cl;
  if (bl >= BB || bl >= nbb || cl >= ncb) return;
  // dt_proj + bias + softplus (tp_model.py:162-163)
  float dot = 0.f;
  const float *dr = dls + bl * R;
#pragma unroll 8
  for (int r = 0; r < R; ++r) dot = fmaf(dr[r], wt[r * (CB + 1) + cl], dot);
  const float dt = softplus_f(dot + ldf(b_dt + c));
  // conv over [history | x] and the history shift (tp_model.py:145-157)
  T *cs = conv_state + ((size_t)b * Es + c) * (K - 1);
  const float xv = ldf(xz + (size_t)b * ld_xz + c);
  float hist[K - 1];
  float acc = conv_b ? ldf(conv_b + c) : 0.f;
#pragma unroll
  for (int j = 0; j < K - 1; ++j) {
    hist[j] = ldf(cs + j);
    acc = fmaf(ldf(conv_w + (size_t)c * K + j), hist[j], acc);
  }
  acc = fmaf(ldf(conv_w + (size_t)c * K + K - 1), xv, acc);
#pragma unroll
  for (int j = 0; j < K - 2; ++j) stf(cs + j, hist[j + 1]);
  stf(cs + K - 2, xv);
  const float xc = silu_f(acc);
  // state update and output (tp_model.py:165-173)
  const float dtx = dt * xc;
  float *hs = ssm_state + ((size_t)b * Es + c) * N;
  const float4 *bc4 = reinterpret_cast<const float4 *>(bcp + (size_t)b * ld_bc);
  const float *a2 = a2s + cl * N;
  float ya[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int q = 0; q < N / 4; ++q) {
    float4 hv = *reinterpret_cast<const float4 *>(hs + 4 * q);
    const float4 B4 = __ldg(bc4 + q), C4 = __ldg(bc4 + N / 4 + q);
    float hh[4] = {hv.x, hv.y, hv.z, hv.w};
    const float Bs[4] = {B4.x, B4.y, B4.z, B4.w}, Cs[4] = {C4.x, C4.y, C4.z, C4.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float dA = ex2_hw(dt * a2[4 * q + u]);
      hh[u] = fmaf(dA, hh[u], Bs[u] * dtx);
      ya[u] = fmaf(Cs[u], hh[u], ya[u]);
    }
    *reinterpret_cast<float4 *>(hs + 4 * q) = make_float4(hh[0], hh[1], hh[2], hh[3]);
  }
  const float zv = ldf(xz + (size_t)b * ld_xz + Es + c);
  const float yv = (ya[0] + ya[1]) + (ya[2] + ya[3]);
  stf(y + (size_t)b * ld_y + c, fmaf(ldf(Dp + c), xc, yv) * silu_f(zv));
}

template <typename T, typename TD, int N, int TPC>
static int launch_scan(const void *xz, int ld_xz, const void *dt_v, int ld_dt, const float *bc, int ld_bc,
                       const void *A_log, const void *Dp, const void *conv_w, const void *conv_b,
                       const void *conv_init, const float *ssm_init, void *y, int ld_y, void *conv_final,
                       float *ssm_final, int B, int L, int Es, cudaStream_t s) {
  constexpr int TL = 16, K = 4;
  using S = ScanSmem<T, TD, N, TPC, TL>;
  constexpr int CB = S::CB;
  auto kern = scan_prefill_kernel<T, TD, N, TPC, TL, K>;
  const TD *dt = (const TD *)dt_v;
  static bool attr_set = false;  // per template instance
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(S)) != cudaSuccess)
      return check_launch("scan_prefill attr");
    attr_set = true;
  }
  const bool vec16 = Es % CB == 0 && aligned16(xz) && aligned16(dt) && aligned16(bc) &&
                     ((size_t)ld_xz * sizeof(T)) % 16 == 0 && ((size_t)ld_dt * sizeof(TD)) % 16 == 0 &&
                     ld_bc % 4 == 0;
  dim3 grid((Es + CB - 1) / CB, B);
  launch_pdl(kern, dim3(grid), dim3(128), sizeof(S), s, (const T *)xz, ld_xz, dt, ld_dt, bc, ld_bc, (const T *)A_log, (const T *)Dp,
                                     (const T *)conv_w, (const T *)conv_b, (const T *)conv_init, ssm_init, (T *)y, ld_y,
                                     (T *)conv_final, ssm_final, L, Es, vec16);
  return check_launch("scan_prefill");
}


// Default number of state pairs per thread whose exponential runs on the FP32 pipe
// (exp2_poly2), by threads per channel; MTP_SCAN_POLY overrides it (0 .. N / (2 TPC)).
constexpr int kPolyPairsTpc1 = 0, kPolyPairsTpc2 = 0, kPolyPairsTpc4 = 0;

// Scratch of the chunked scan's state pass ([B][NC][Es][N+1] fp32), per device, grown on
// demand (outside stream capture: the prefill is not captured).
static float *scan_chunk_scratch(size_t bytes) {
  constexpr int MAXD = 64;
  static float *ptr[MAXD] = {};
  static size_t cap[MAXD] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAXD) return nullptr;
  if (cap[dev] < bytes) {
    if (ptr[dev]) {
      cudaDeviceSynchronize();
      cudaFree(ptr[dev]);
    }
    ptr[dev] = nullptr;
    cap[dev] = 0;
    if (cudaMalloc(&ptr[dev], bytes) != cudaSuccess) return nullptr;
    cap[dev] = bytes;
  }
  return ptr[dev];
}

template <typename T, typename TD, int N, int TPC, int NPP, int MINB>
static int launch_scan_xc(const void *xc, int ld_xc, const void *xz, int ld_xz, const void *dt_v, int ld_dt,
                          const float *bc, int ld_bc, const void *A_log, const void *Dp, const void *conv_init,
                          const float *ssm_init, void *y, int ld_y, void *conv_final, float *ssm_final, int B, int L,
                          int Es, int nc, cudaStream_t s) {
  constexpr int TL = 16, K = 4;
  using S = ScanXcSmem<T, TD, N, TPC, TL>;
  constexpr int CB = S::CB;
  auto kern = scan_xc_kernel<T, TD, N, TPC, TL, K, NPP, MINB, false>;
  auto kern_st = scan_xc_kernel<T, TD, N, TPC, TL, K, NPP, MINB, true>;
  const TD *dt = (const TD *)dt_v;
  static bool attr_set = false;  // per template instance
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(S)) != cudaSuccess ||
        cudaFuncSetAttribute(kern_st, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(S)) != cudaSuccess)
      return check_launch("scan_prefill_xc attr");
    attr_set = true;
  }
  const bool vec16 = Es % CB == 0 && aligned16(xc) && aligned16(xz) && aligned16(dt) && aligned16(bc) &&
                     ((size_t)ld_xc * sizeof(T)) % 16 == 0 && ((size_t)ld_xz * sizeof(T)) % 16 == 0 &&
                     ((size_t)Es * sizeof(T)) % 16 == 0 && ((size_t)ld_dt * sizeof(TD)) % 16 == 0 && ld_bc % 4 == 0;
  // sequence chunks of Lc positions (a multiple of the token tile)
  int Lc = L, NC = 1;
  if (nc > 1) {
    Lc = (L + nc - 1) / nc;
    Lc = (Lc + TL - 1) / TL * TL;
    NC = (L + Lc - 1) / Lc;
  }
  float *io = nullptr;
  if (NC > 1) {
    io = scan_chunk_scratch((size_t)B * NC * Es * (N + 1) * sizeof(float));
    if (!io) return fail(MTP_ERR_CUDA, "could not allocate the chunked scan's state scratch");
    dim3 g1((Es + CB - 1) / CB, B, NC - 1);  // the last chunk's end state is not needed
    launch_pdl(kern_st, dim3(g1), dim3(128), sizeof(S), s, (const T *)xc, ld_xc, (const T *)xz, ld_xz, dt, ld_dt, bc,
               ld_bc, (const T *)A_log, (const T *)Dp, (const T *)conv_init, ssm_init, (T *)y, ld_y, (T *)conv_final,
               ssm_final, L, Es, vec16, Lc, NC, io);
    int rc = check_launch("scan_prefill_xc states");
    if (rc) return rc;
  }
  dim3 grid((Es + CB - 1) / CB, B, NC);
  launch_pdl(kern, dim3(grid), dim3(128), sizeof(S), s, (const T *)xc, ld_xc, (const T *)xz, ld_xz, dt, ld_dt, bc,
             ld_bc, (const T *)A_log, (const T *)Dp, (const T *)conv_init, ssm_init, (T *)y, ld_y, (T *)conv_final,
             ssm_final, L, Es, vec16, Lc, NC, io);
  return check_launch("scan_prefill_xc");
}

// Picks the instance for (threads per channel, polynomial pairs, CTAs per SM).  The
// FP32-pipe exponential did not pay on B200 (1.4b TP=1 shard, 32 x 1024: 0.69 ms with no
// polynomial pairs, 0.71 / 0.77 / 0.83 / 0.90 ms with 1 / 2 / 3 / 4 of 8), so every
// default is 0; bf16 models with bf16 dt and d_state 16 also build one polynomial split
// per width (MTP_SCAN_POLY, tests) and, for one thread per channel, 4, 5 or 6 resident
// CTAs per SM (MTP_SCAN_OCC; 4, the default, measured best: 0.688 / 0.691 / 0.690 ms).
template <typename T, typename TD, int N, int TPC>
static int scan_xc_npp(int npp, int occ, const void *xc, int ld_xc, const void *xz, int ld_xz, const void *dt,
                       int ld_dt, const float *bc, int ld_bc, const void *A_log, const void *Dp, const void *conv_init,
                       const float *ssm_init, void *y, int ld_y, void *conv_final, float *ssm_final, int B, int L,
                       int Es, int nc, cudaStream_t s) {
#define MTP_SXC(P, OCC)                                                                                          \
  return launch_scan_xc<T, TD, N, TPC, P, OCC>(xc, ld_xc, xz, ld_xz, dt, ld_dt, bc, ld_bc, A_log, Dp, conv_init, \
                                               ssm_init, y, ld_y, conv_final, ssm_final, B, L, Es, nc, s)
  constexpr int NP = N / TPC / 2;
  constexpr int DEF = TPC == 1 ? kPolyPairsTpc1 : TPC == 2 ? kPolyPairsTpc2 : kPolyPairsTpc4;
  constexpr int D0 = DEF < NP ? DEF : NP;
  constexpr int OCC0 = TPC == 1 ? 4 : 6;
  constexpr int P1 = NP >= 2 ? 2 : 1;
  constexpr bool ALL = std::is_same<T, __nv_bfloat16>::value && std::is_same<TD, __nv_bfloat16>::value && N == 16;
  if constexpr (ALL) {
    if (npp == P1) MTP_SXC(P1, OCC0);
    if constexpr (TPC == 1) {
      if (npp == D0 && occ == 5) MTP_SXC(D0, 5);
      if (npp == D0 && occ == 6) MTP_SXC(D0, 6);
    }
  }
  MTP_SXC(D0, OCC0);
#undef MTP_SXC
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
  cudaStream_t s = (cudaStream_t)stream;
  const size_t es_b = dtype == MTP_F32 ? 4 : 2;
  const int V = (int)(16 / es_b);
  const bool vec = Es % V == 0 && aligned16(xz) && aligned16(xc) && (ld_xz * es_b) % 16 == 0 && (ld_xc * es_b) % 16 == 0;
  if (vec) {
    // B200, 1.4b TP=1 shard: all of a thread's loads issued first, 8 positions per thread
    // (0.121 ms, the default); the 64-position direct loop (MTP_CONV_KERNEL=direct, 0.170 ms);
    // the input tile staged in shared memory (MTP_CONV_STAGED=1, 0.234 ms)
    constexpr int TT = 64, NTH = 32;
    const int groups = Es / V;
    const bool wvec = aligned16(conv_w) && (conv_b == nullptr || aligned16(conv_b));
    static const bool staged = [] {
      const char *e = getenv("MTP_CONV_STAGED");
      return e && e[0] == '1';
    }();
    // default: all of a thread's loads issued first (MTP_CONV_KERNEL=direct: the
    // 64-position loop above)
    const char *ek = getenv("MTP_CONV_KERNEL");  // read per call: tests switch it
    const bool direct = ek && !strcmp(ek, "direct");
    const char *ep = getenv("MTP_CONV_P");  // positions per thread: 8 (128 registers, 4 CTAs per SM) or 16
    const int pos = ep && atoi(ep) == 16 ? 16 : 8;
    if (!staged && !direct) {
      constexpr int NB = 128;
      dim3 g2((groups + NB - 1) / NB, (L + pos - 1) / pos, B);
      if (pos == 16)
        MTP_DISPATCH_FB(dtype, T,
            launch_pdl(conv1d_silu_batch_kernel<T, 4, 16>, dim3(g2), dim3(NB), 0, s, (const T *)xz, ld_xz,
                       (const T *)conv_w, (const T *)conv_b, (const T *)hist, (T *)xc, ld_xc, L, Es, wvec));
      else
        MTP_DISPATCH_FB(dtype, T,
            launch_pdl(conv1d_silu_batch_kernel<T, 4, 8>, dim3(g2), dim3(NB), 0, s, (const T *)xz, ld_xz,
                       (const T *)conv_w, (const T *)conv_b, (const T *)hist, (T *)xc, ld_xc, L, Es, wvec));
      return check_launch("conv1d_silu");
    }
    dim3 grid((groups + (staged ? NTH : 64) - 1) / (staged ? NTH : 64), (L + TT - 1) / TT, B);
    if (staged) {
      const size_t smem = (size_t)(TT + 3) * NTH * 16;
      MTP_DISPATCH_FB(dtype, T, {
        auto kern = conv1d_silu_smem_kernel<T, 4, TT, NTH>;
        static bool attr = false;
        if (!attr) {
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
          attr = true;
        }
        launch_pdl(kern, dim3(grid), dim3(NTH), smem, s, (const T *)xz, ld_xz, (const T *)conv_w, (const T *)conv_b,
                   (const T *)hist, (T *)xc, ld_xc, L, Es, wvec);
      });
      return check_launch("conv1d_silu");
    }
    MTP_DISPATCH_FB(dtype, T,
        launch_pdl(conv1d_silu_vec_kernel<T, 4, TT>, dim3(grid), dim3(64), 0, s, (const T *)xz, ld_xz, (const T *)conv_w,
                                                              (const T *)conv_b, (const T *)hist, (T *)xc, ld_xc, L, Es, wvec));
    return check_launch("conv1d_silu");
  }
  constexpr int TT = 8;
  dim3 grid((Es + 127) / 128, (L + TT - 1) / TT, B);
  MTP_DISPATCH_FB(dtype, T,
      launch_pdl(conv1d_silu_kernel<T, 4, TT>, dim3(grid), dim3(128), 0, s, (const T *)xz, ld_xz, (const T *)conv_w,
                                                         (const T *)conv_b, (const T *)hist, (T *)xc, ld_xc, L, Es));
  return check_launch("conv1d_silu");
}

int mtp_scan_prefill(const void *xz, int ld_xz, const void *dt, int ld_dt, int dt_dtype, const float *bc, int ld_bc,
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
  MTP_REQUIRE(dt_dtype == MTP_F32 || dt_dtype == dtype, "dt must be F32 or the model dtype");
  MTP_REQUIRE(dt_dtype == MTP_F32 || (ld_dt % 2 == 0 && Es % 2 == 0), "bf16 dt rows need even Es and ld_dt");
  if (B == 0 || L == 0) return MTP_OK;
  cudaStream_t s = (cudaStream_t)stream;
  // threads per channel: one (all 16 states in registers) unless there are too few
  // (sequence, channel) pairs to occupy the SMs.  B200, 32 x 1024 tokens: 2048
  // channels 0.54 / 0.70 / 0.97 ms for 1 / 2 / 4 threads, 1024: 0.35 / 0.53 / 0.58,
  // 512: 0.31 / 0.29 / 0.41.
  const long pairs = (long)B * Es;
  const int sms = num_sms();
  int tpc = pairs >= (long)sms * 128 ? 1 : (pairs >= (long)sms * 32 ? 2 : 4);
  // tuning override: MTP_SCAN_TPC = 1, 2 or 4 threads per channel
  if (const char *env = getenv("MTP_SCAN_TPC")) {
    const int v = atoi(env);
    if (v == 1 || v == 2 || v == 4) tpc = v;
  }
#define MTP_SCAN_CASE(TT, TDD, NN, TP)                                                                     \
  return launch_scan<TT, TDD, NN, TP>(xz, ld_xz, dt, ld_dt, bc, ld_bc, A_log, Dp, conv_w, conv_b, conv_init, \
                                      ssm_init, y, ld_y, conv_final, ssm_final, B, L, Es, s)
  using bf16 = __nv_bfloat16;
  if (dtype == MTP_F32) {
    if (N == 16) { if (tpc == 1) MTP_SCAN_CASE(float, float, 16, 1); if (tpc == 2) MTP_SCAN_CASE(float, float, 16, 2); MTP_SCAN_CASE(float, float, 16, 4); }
    MTP_SCAN_CASE(float, float, 8, 2);
  } else if (dtype == MTP_BF16 && dt_dtype == MTP_F32) {
    if (N == 16) { if (tpc == 1) MTP_SCAN_CASE(bf16, float, 16, 1); if (tpc == 2) MTP_SCAN_CASE(bf16, float, 16, 2); MTP_SCAN_CASE(bf16, float, 16, 4); }
    MTP_SCAN_CASE(bf16, float, 8, 2);
  } else if (dtype == MTP_BF16) {
    if (N == 16) { if (tpc == 1) MTP_SCAN_CASE(bf16, bf16, 16, 1); if (tpc == 2) MTP_SCAN_CASE(bf16, bf16, 16, 2); MTP_SCAN_CASE(bf16, bf16, 16, 4); }
    MTP_SCAN_CASE(bf16, bf16, 8, 2);
  }
#undef MTP_SCAN_CASE
  return fail(MTP_ERR_UNSUPPORTED, "scan_prefill: dtype must be F32 or BF16");
}

int mtp_scan_prefill_xc(const void *xc, int ld_xc, const void *xz, int ld_xz, const void *dt, int ld_dt, int dt_dtype,
                        const float *bc, int ld_bc, const void *A_log, const void *Dp, const void *conv_init,
                        const float *ssm_init, void *y, int ld_y, void *conv_final, float *ssm_final, int B, int L,
                        int Es, int N, int K, int dtype, void *stream) {
  MTP_REQUIRE(xc && xz && dt && bc && A_log && Dp && y && conv_final && ssm_final, "null pointer");
  MTP_REQUIRE(B >= 0 && L >= 0 && Es > 0, "bad sizes");
  MTP_REQUIRE(K == 4, "only d_conv == 4 is built");
  MTP_REQUIRE(N == 16 || N == 8, "d_state must be 8 or 16");
  MTP_REQUIRE(ld_xc >= Es && ld_xz >= 2 * Es && ld_dt >= Es && ld_bc >= 2 * N && ld_y >= Es,
              "leading dimensions too small");
  MTP_REQUIRE(dtype == MTP_F32 || dtype == MTP_BF16, "dtype must be F32 or BF16");
  const size_t es = dtype == MTP_F32 ? 4 : 2;
  // 4-byte cp.async granules: element pairs must be 4-byte aligned
  MTP_REQUIRE(aligned(xc, 4) && aligned(xz, 4) && aligned(dt, 4) && aligned(bc, 4), "inputs must be 4-byte aligned");
  MTP_REQUIRE(es == 4 || (ld_xz % 2 == 0 && ld_xc % 2 == 0 && Es % 2 == 0), "bf16 rows need even Es and strides");
  MTP_REQUIRE(dt_dtype == MTP_F32 || dt_dtype == dtype, "dt must be F32 or the model dtype");
  MTP_REQUIRE(dt_dtype == MTP_F32 || (ld_dt % 2 == 0 && Es % 2 == 0), "bf16 dt rows need even Es and ld_dt");
  if (B == 0 || L == 0) return MTP_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const long pairs = (long)B * Es;
  const int sms = num_sms();
  int tpc = pairs >= (long)sms * 128 ? 1 : (pairs >= (long)sms * 32 ? 2 : 4);
  if (const char *env = getenv("MTP_SCAN_TPC")) {
    const int v = atoi(env);
    if (v == 1 || v == 2 || v == 4) tpc = v;
  }
  if (N == 8) tpc = 2;
  int npp = tpc == 1 ? kPolyPairsTpc1 : tpc == 2 ? kPolyPairsTpc2 : kPolyPairsTpc4;
  if (const char *env = getenv("MTP_SCAN_POLY")) npp = atoi(env);
  if (npp < 0) npp = 0;
  int occ = 0;
  if (const char *env = getenv("MTP_SCAN_OCC")) occ = atoi(env);
  // sequence chunks when few recurrences run per SM (B x Es up to 8192, e.g. 8 sequences x
  // 640 channels) and the sequences are long: the state pass doubles the SFU work of all but
  // the last chunk but multiplies the parallelism.  B200, 8 x 8192 x 640 (2.8b TP=8 shard):
  // 1.275 ms unchunked, 0.620 / 0.625 / 0.450 ms with 4 / 8 / 16 chunks; 32 x 1024 x 512 (1.4b
  // TP=8): 0.187 / 0.184 / 0.193 ms with 1 / 2 / 4, so no chunks there.  MTP_SCAN_CHUNKS=n forces n.
  int nc = 1;
  if (pairs <= 8192 && L >= 2048) nc = L / 512 < 16 ? L / 512 : 16;
  if (const char *env = getenv("MTP_SCAN_CHUNKS")) nc = atoi(env);
  if (nc < 1) nc = 1;
#define MTP_SXC_CASE(TT, TDD, NN, TP)                                                                          \
  return scan_xc_npp<TT, TDD, NN, TP>(npp, occ, xc, ld_xc, xz, ld_xz, dt, ld_dt, bc, ld_bc, A_log, Dp, conv_init, \
                                      ssm_init, y, ld_y, conv_final, ssm_final, B, L, Es, nc, s)
  using bf16 = __nv_bfloat16;
  if (dtype == MTP_F32) {
    if (N == 16) { if (tpc == 1) MTP_SXC_CASE(float, float, 16, 1); if (tpc == 2) MTP_SXC_CASE(float, float, 16, 2); MTP_SXC_CASE(float, float, 16, 4); }
    MTP_SXC_CASE(float, float, 8, 2);
  } else if (dt_dtype == MTP_F32) {
    if (N == 16) { if (tpc == 1) MTP_SXC_CASE(bf16, float, 16, 1); if (tpc == 2) MTP_SXC_CASE(bf16, float, 16, 2); MTP_SXC_CASE(bf16, float, 16, 4); }
    MTP_SXC_CASE(bf16, float, 8, 2);
  } else {
    if (N == 16) { if (tpc == 1) MTP_SXC_CASE(bf16, bf16, 16, 1); if (tpc == 2) MTP_SXC_CASE(bf16, bf16, 16, 2); MTP_SXC_CASE(bf16, bf16, 16, 4); }
    MTP_SXC_CASE(bf16, bf16, 8, 2);
  }
#undef MTP_SXC_CASE
}

int mtp_exp2_fma(const float *x, float *out, int n, void *stream) {
  MTP_REQUIRE(x && out && n >= 0, "bad arguments");
  if (n == 0) return MTP_OK;
  const int pairs = (n + 1) / 2;
  launch_pdl(exp2_fma_kernel, dim3((pairs + 255) / 256), dim3(256), 0, (cudaStream_t)stream, x, out, n);
  return check_launch("exp2_fma");
}

int mtp_scan_prefill_fused(const void *xz, int ld_xz, const void *dt_low, int ld_dl, const void *W_dt,
                           const void *b_dt, const float *bc, int ld_bc, const void *A_log, const void *Dp,
                           const void *conv_w, const void *conv_b, const void *conv_init, const float *ssm_init,
                           void *y, int ld_y, void *conv_final, float *ssm_final, int B, int L, int Es, int N, int R,
                           int K, void *stream) {
  MTP_REQUIRE(xz && dt_low && W_dt && b_dt && bc && A_log && Dp && conv_w && y && conv_final && ssm_final,
              "null pointer");
  MTP_REQUIRE(B >= 0 && L >= 0 && Es > 0 && R > 0, "bad sizes");
  MTP_REQUIRE(K == 4 && N == 16, "the fused scan is built for d_conv 4, d_state 16");
  MTP_REQUIRE(Es % 128 == 0, "the fused scan needs d_inner per rank divisible by 128");
  MTP_REQUIRE(R % 8 == 0 && R <= 256 && ld_dl % 8 == 0 && ld_dl >= R, "dt_rank must be a multiple of 8, at most 256");
  MTP_REQUIRE(aligned16(xz) && aligned16(dt_low) && aligned16(W_dt) && aligned16(bc) && ld_xz % 8 == 0 && ld_bc % 4 == 0 &&
                  ld_bc >= 2 * N && ld_xz >= 2 * Es && ld_y >= Es,
              "fused scan needs 16-byte aligned rows");
  if (B == 0 || L == 0) return MTP_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const int ka = (R + 63) / 64;
#define MTP_FS(KA_)                                                                                          \
  return launch_scan_fused<KA_>(xz, ld_xz, dt_low, ld_dl, W_dt, b_dt, bc, ld_bc, A_log, Dp, conv_w, conv_b, \
                                conv_init, ssm_init, y, ld_y, conv_final, ssm_final, B, L, Es, R, s)
  if (ka == 1) MTP_FS(1);
  if (ka == 2) MTP_FS(2);
  if (ka == 3) MTP_FS(3);
  MTP_FS(4);
#undef MTP_FS
}

int mtp_scan_status(int *status) {
  MTP_REQUIRE(status, "null argument");
  int *w = scan_err_word();
  if (!w) return fail(MTP_ERR_CUDA, "no status word");
  if (cudaMemcpy(status, w, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return fail(MTP_ERR_CUDA, "read status");
  return MTP_OK;
}

int mtp_step(const void *xz, int ld_xz, const void *dt_low, int ld_dl, const void *W_dt, const void *b_dt,
             const float *bc, int ld_bc, const void *A_log, const void *Dp, const void *conv_w, const void *conv_b,
             void *conv_state, float *ssm_state, void *y, int ld_y, int B, int Es, int N, int R, int K, int dtype,
             void *stream) {
  MTP_REQUIRE(xz && dt_low && W_dt && b_dt && bc && A_log && Dp && conv_w && conv_state && ssm_state && y,
              "null pointer");
  MTP_REQUIRE(K == 4, "only d_conv == 4 is built");
  MTP_REQUIRE(N == 16 || N == 8, "d_state must be 8 or 16");
  MTP_REQUIRE(B >= 0 && B <= 1024 && Es > 0 && R > 0, "bad sizes");
  MTP_REQUIRE(aligned16(ssm_state) && aligned16(bc) && ld_bc % 4 == 0, "ssm_state / bc must be 16-byte aligned");
  if (B == 0) return MTP_OK;
  constexpr int CB = 32;
  const int BB = B >= 8 ? 8 : (B >= 4 ? 4 : (B >= 2 ? 2 : 1));
  const size_t smem = ((size_t)R * (CB + 1) + (size_t)BB * R + (size_t)CB * N) * sizeof(float);
  MTP_REQUIRE(smem <= 200 * 1024, "dt_rank too large for the step kernel");
  cudaStream_t s = (cudaStream_t)stream;
  dim3 grid((Es + CB - 1) / CB, (B + BB - 1) / BB);
#define MTP_STEP_CASE(TT, NN)                                                                               \
  do {                                                                                                     \
    auto kern = step_kernel<TT, NN, 4>;                                                                    \
    static bool attr_set = false;                                                                          \
    if (!attr_set) {                                                                                       \
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);                 \
      attr_set = true;                                                                                     \
    }                                                                                                      \
    launch_pdl(kern, dim3(grid), dim3(256), smem, s, (const TT *)xz, ld_xz, (const TT *)dt_low, ld_dl, (const TT *)W_dt,       \
                                 (const TT *)b_dt, bc, ld_bc, (const TT *)A_log, (const TT *)Dp,          \
                                 (const TT *)conv_w, (const TT *)conv_b, (TT *)conv_state, ssm_state,     \
                                 (TT *)y, ld_y, B, Es, R, BB);                                             \
    return check_launch("step");                                                                           \
  } while (0)
  if (dtype == MTP_F32) { if (N == 16) MTP_STEP_CASE(float, 16); MTP_STEP_CASE(float, 8); }
  if (dtype == MTP_BF16) { if (N == 16) MTP_STEP_CASE(__nv_bfloat16, 16); MTP_STEP_CASE(__nv_bfloat16, 8); }
#undef MTP_STEP_CASE
  return fail(MTP_ERR_UNSUPPORTED, "step: dtype must be F32 or BF16");
}

}  // extern "C"
