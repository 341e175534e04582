// Element arithmetic of the reductions' wire formats (mamba_lite/tp_utils.py), shared by
// the reduction kernels (comm.cu) and the x_proj GEMM epilogue that writes the wire
// directly (gemm_tc.cu), so both produce the same bytes.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include "../../include/mtp.h"

namespace mtp {

// Per-row int8 quantisation (tp_utils.py:111-112), IEEE divide and round-half-even.
__device__ __forceinline__ float row_scale(float amax) { return __fdiv_rn(fmaxf(amax, 1e-8f), 127.0f); }
__device__ __forceinline__ int quant1(float x, float scale) {
  float r = rintf(__fdiv_rn(x, scale));
  r = fminf(fmaxf(r, -127.0f), 127.0f);
  return (int)r;
}
__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  return (uint32_t)(a & 0xff) | ((uint32_t)(b & 0xff) << 8) | ((uint32_t)(c & 0xff) << 16) | ((uint32_t)(d & 0xff) << 24);
}
__device__ __forceinline__ float unpack_i8(uint32_t w, int i) { return (float)(int8_t)((w >> (8 * i)) & 0xffu); }

// Round to the collective's return dtype: the reference's reductions return the
// model dtype (tp_utils.py:42, :131), so a bf16 model sees bf16-rounded sums.
__device__ __forceinline__ float rnd_rdt(float x, int rdt) {
  return rdt == MTP_BF16 ? __bfloat162float(__float2bfloat16_rn(x)) : x;
}

// World size 1: one value's int8 round trip as the rank-ordered sum from zero
// (tp_utils.py:126-130), and the fp16 round trip (tp_utils.py:37-42).
__device__ __forceinline__ float dq1(float x, float s) { return __fadd_rn(0.f, __fmul_rn((float)quant1(x, s), s)); }
__device__ __forceinline__ float h1(float x) { return __half2float(__float2half_rn(x)); }

// Outputs of the x_proj GEMM whose epilogue performs AllReduce #1's first half
// (gemm_tc_xproj_wire): world size 1 writes dt_low / B|C directly; world size > 1 writes
// the wire rows into every rank's receive slot and raises this CTA's phase-0 flag.
struct XprojWire {
  int wmode, rdt, R, dt_dtype, ws, rank;
  void *dt_low;                 // world size 1: [M, R] in dt_dtype
  float *bc;                    // world size 1: [M, N - R] fp32
  char *wslot[8];               // rank k's receive slot for this rank (half 0)
  unsigned long long whalf;     // bytes from half 0 to half 1 of the slots
  uint32_t *wflag[8];           // rank k's phase-0 flag word of this rank's CTA 0 (CTA j at + j)
  const uint32_t *wepoch;       // this rank's epoch word of the site
};

int gemm_tc_xproj_wire(const void *A, const void *B, int M, int N, int K, int lda, int ldb, const XprojWire &w,
                       int *grid_out, cudaStream_t stream);

}  // namespace mtp
