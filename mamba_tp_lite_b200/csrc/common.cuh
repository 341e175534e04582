// Shared helpers for libmtp.so (sm_100a only).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <atomic>
#include <string>

#include "../../include/mtp.h"

namespace mtp {

// ----------------------------------------------------------------- host errors
void set_error(const std::string &msg);
int fail(int code, const std::string &msg);
int check_launch(const char *what);
extern std::atomic<uint64_t> g_launches;
inline void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
int num_sms();

#define MTP_REQUIRE(cond, msg)                                   \
  do {                                                           \
    if (!(cond)) return ::mtp::fail(MTP_ERR_ARG, std::string(__func__) + ": " + (msg)); \
  } while (0)

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
inline int ceil_div(long a, long b) { return (int)((a + b - 1) / b); }

// ----------------------------------------------------------------- element access
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float ld(const float *p) { return *p; }
  static __device__ __forceinline__ void st(float *p, float v) { *p = v; }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float ld(const __nv_bfloat16 *p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ void st(__nv_bfloat16 *p, float v) { *p = __float2bfloat16_rn(v); }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float ld(const __half *p) { return __half2float(*p); }
  static __device__ __forceinline__ void st(__half *p, float v) { *p = __float2half_rn(v); }
};

template <typename T> __device__ __forceinline__ float ldf(const T *p) { return Elem<T>::ld(p); }
template <typename T> __device__ __forceinline__ void stf(T *p, float v) { Elem<T>::st(p, v); }

// torch semantics, fp32.  Library expf / log1pf are called (not reimplemented).
__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float softplus_f(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

// softplus(x) = max(x, 0) + log1p(exp(-|x|)), torch's threshold 20.  log1p(u) for
// u in (0, 1] by Goldberg's identity log1p(u) = log(1+u) * u / ((1+u) - 1), which
// keeps the relative accuracy of the hardware logarithm for small u.
// Written without branches (selects only) so a thread's many independent
// elements overlap their MUFU latencies.
__device__ __forceinline__ float softplus_fast(float x) {
  const float u = __expf(-fabsf(x));
  const float w = 1.0f + u;
  const float lg = __logf(w) * __fdividef(u, w - 1.0f);  // w == 1: not selected below
  const float r = fmaxf(x, 0.f) + ((w == 1.0f) ? u : lg);
  return x > 20.f ? x : r;
}


// softplus with two MUFU operations (ex2, lg2) instead of three: max(x, 0) + log1p(t),
// t = e^-|x| in (0, 1]; log1p(t) is the hardware log of 1 + t for t >= 2^-12 (absolute
// error about 6e-8, so relative error <= 2.5e-4 there) and t - t^2/2 below (relative error
// < 2^-25).  For outputs rounded to bf16 (relative step 2^-8) after the tensor-core GEMMs.
__device__ __forceinline__ float softplus_bf16out(float x) {
  const float t = __expf(-fabsf(x));
  const float small = t * fmaf(-0.5f, t, 1.0f);
  const float l = __logf(1.0f + t);
  const float r = fmaxf(x, 0.f) + (t < 2.44140625e-4f ? small : l);
  return x > 20.f ? x : r;
}

// SiLU with the hardware exponential and a fast divide, x / (1 + e^-x).
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// ----------------------------------------------------------------- timing / waits
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// ----------------------------------------------------------------- programmatic dependent launch
// Every kernel of the library is launched with programmatic stream serialization
// allowed, so the next kernel's launch and prologue overlap the tail of the
// current one.  Each kernel therefore executes MTP_PDL_WAIT() before its first
// global-memory access (it returns once the previous kernel has completed and
// its writes are visible) and MTP_PDL_TRIGGER() to let its dependent launch.
// Without a programmatic predecessor both are no-ops.  MTP_PDL=0 turns it off.
#define MTP_PDL_WAIT() asm volatile("griddepcontrol.wait;" ::: "memory")
#define MTP_PDL_TRIGGER() asm volatile("griddepcontrol.launch_dependents;" ::: "memory")

bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// dispatch on a runtime dtype code
#define MTP_DISPATCH_FB(code, T, ...)                                       \
  do {                                                                      \
    if ((code) == MTP_F32) { using T = float; __VA_ARGS__; }                \
    else if ((code) == MTP_BF16) { using T = __nv_bfloat16; __VA_ARGS__; } \
    else return ::mtp::fail(MTP_ERR_UNSUPPORTED, "dtype must be F32 or BF16"); \
  } while (0)

}  // namespace mtp
