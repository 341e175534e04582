// Persistent decode: one cooperative launch runs a whole single-token step of the
// language model (every layer), replacing the per-layer kernel chain of a step.
//
// Reference behaviour restated (mamba_lite):
//   embedding gather                   tp_model.py:318, model.py:348
//   per layer (TPMambaMixer.step)      tp_model.py:137-179
//     in_proj, conv state shift + conv + SiLU     :141-157
//     x_proj -> AllReduce #1 -> dt | B | C         :159-161
//     dt_proj + softplus, state update, C.h + D.x, gate   :162-173
//     out_proj -> AllReduce #2 (+ bias)            :175-178
//   block RMSNorm + residual           tp_model.py:259-262, model.py:130-135
//   norm_f after the last layer        tp_model.py:321
// The collectives keep the wire formats and rank-ordered sums of tp_utils.py
// (fp32 :23-28, fp16 :31-42, int8 per token :103-131) over the comm context's
// NVLink peer slots, and every reduced value is rounded to the model dtype.
//
// Grid: one 256-thread CTA per SM (cooperative launch).  Phases per layer:
//   P1  in_proj row tiles (16 rows x all tokens, mma.sync bf16, fp32 accumulate) with
//       the conv as epilogue: x|z rounded to bf16, conv history shifted, xc = SiLU(conv)
//   P2  x_proj row tiles, K split over CTAs -> fp32 partials
//   P3  owner CTA b sums row b's partials in split order, runs AllReduce #1 for the row
//       (push its wire row to every rank, wait for theirs, rank-ordered sum) and publishes
//       the reduced row with a per-row flag; no grid barrier between P3 and P4
//   P4  16-channel tiles: wait for every token's flag, dt_proj as an MMA row tile over the
//       bf16 dt_low tokens, softplus, state update with 16/SPLIT states per thread
//       (SPLIT chosen so the tile's 16 x B pairs fill the CTA), y = (C.h + D xc) SiLU(z)
//   P5  out_proj row tiles -> fp32 partials
//   P6  owner CTA b: sum, AllReduce #2, + bias, residual (kept in the owner's registers
//       for the whole step), next RMSNorm
// No grid barrier: each phase waits (bounded) only for the counters / per-row flags of
// the data it reads (see "dependency counters").  Before doing its part of a phase,
// each CTA asks L2 to prefetch (cp.async.bulk.prefetch.L2) the weight rows of the units
// it will process one or two phases later, so HBM streams across the barriers.
// Every wait is bounded: on expiry the kernel records MTP_ERR_TIMEOUT, raises the abort
// word, and every CTA returns at its next wait.
#include <cstdlib>
#include <cstring>
#include <vector>
#include "common.cuh"
#include "comm_dev.cuh"

namespace mtp {

using bf16 = __nv_bfloat16;

constexpr int DT = 256;  // threads per CTA
constexpr int DW = 8;    // warps per CTA
constexpr int DN = 16;   // d_state handled by the kernel
constexpr int DK = 4;    // d_conv handled by the kernel
constexpr int XPAD = 32; // bf16 elements of padding per staged token row (bank spread)
static_assert(DT == 16 * DN, "one thread per (channel, state) of a 16-channel tile");

struct DecLayer {
  const bf16 *norm_w, *in_w, *in_b, *conv_w, *conv_b, *x_w, *dt_w, *dt_b, *A_log, *Dp, *out_w, *out_b;
  int mode_x, mode_out;
};
struct DecCache {
  bf16 *conv;  // [B][Es][K-1]
  float *ssm;  // [B][Es][N]
};

struct DecParams {
  const DecLayer *layers;
  const DecCache *cache;
  int n_layer;
  const bf16 *norm_f, *emb;
  const int64_t *ids;
  bf16 *normed;      // [B][D]
  bf16 *xcT, *zT, *yT;
  float *xcf;        // [B][Es]
  float *pxp;        // [KCx][B][NX]
  float *xd;         // [B][NX] reduced x_proj rows (dt_low | B | C), published per row
  unsigned *lflags;  // [B] per-row publication flags (value = local epoch)
  unsigned *lepoch;  // local epoch: one per layer, advanced at the end of each launch
  float *pop;        // [KCo][B][D]
  unsigned *bar;     // [0] unused, [1] exits, [2] abort
  unsigned *cnt;     // dependency counters (layout: see cnt_* below), zero between launches
  int ncnt;
  int *err;
  unsigned long long *trace;  // NULL, or [2 + 5 n_layer] globaltimer stamps of CTA 0 (phase ends)
  int B, D, Es, R, NX, KCx, KCo, chunk_x, chunk_o, xstride;
  float eps;
  int has_comm;
  int prefetch;      // issue the L2 bulk prefetches (MTP_DECODE_PREFETCH=0 turns them off)
  CommDev cv;
  unsigned long long timeout_ns;
};

// ----------------------------------------------------------------- small device helpers
__device__ __forceinline__ uint32_t ld_acquire_gpu(const unsigned *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint4 ldg_stream(const bf16 *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Prefetch [p, p + bytes) into L2 in 16 KB pieces, spread over the lanes of one warp.
// p must be 16-byte aligned and bytes a multiple of 16.
__device__ __forceinline__ void prefetch_range(const void *p, size_t bytes, int lane) {
  constexpr size_t PIECE = 16384;
  const char *c = static_cast<const char *>(p);
  for (size_t o = (size_t)lane * PIECE; o < bytes; o += 32 * PIECE) {
    const size_t n = bytes - o < PIECE ? bytes - o : PIECE;
    prefetch_l2(c + o, (uint32_t)n);
  }
}

__device__ __forceinline__ float bf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
__device__ __forceinline__ float ldbf(const bf16 *p) { return __bfloat162float(*p); }
__device__ __forceinline__ float ldcg_bf(const bf16 *p) {
  return __bfloat162float(__ushort_as_bfloat16(__ldcg(reinterpret_cast<const unsigned short *>(p))));
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Block-wide sum (or max) with a fixed combination order; every thread gets the result.
__device__ __forceinline__ float block_allreduce(float v, float *red32, bool is_max) {
  for (int o = 16; o; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, w) : v + w;
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red32[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red32[0];
  for (int i = 1; i < DW; ++i) r = is_max ? fmaxf(r, red32[i]) : r + red32[i];
  return r;
}

__device__ __forceinline__ float q_scale(float amax) { return __fdiv_rn(fmaxf(amax, 1e-8f), 127.0f); }
__device__ __forceinline__ int q_one(float x, float s) {
  return (int)fminf(fmaxf(rintf(__fdiv_rn(x, s)), -127.0f), 127.0f);
}

// ----------------------------------------------------------------- dependency counters
// The phases of a layer hand data to each other through counters and per-row flags
// instead of grid barriers: a producer CTA finishes a tile (all threads, __syncthreads),
// then thread 0 fences and adds to the tile's counter; a consumer's thread 0 spins
// (acquire, bounded by timeout_ns, abandoning on the abort word) until the counter
// reaches the layer's target, then the CTA reads the data with L2 (.cg) loads.  Every
// CTA runs the phases in the same order and only waits for work of earlier phases of
// co-resident CTAs (cooperative launch), so no wait can be part of a cycle.  Counters
// count cumulatively over the layers of a launch and are reset by the last CTA to exit.
//   cnt[0, KCx)           in_proj x tiles done per x_proj K chunk   (target (l+1) x tiles in chunk)
//   cnt[KCx]              in_proj z tiles done                     (target (l+1) x Es/16)
//   cnt[KCx+1]            x_proj units done                        (target (l+1) x units)
//   cnt[KCx+2, +KCo)      step tiles done per out_proj K chunk      (target (l+1) x tiles in chunk)
//   cnt[KCx+2+KCo]        out_proj units done                      (target (l+1) x units)
//   cnt[KCx+3+KCo, +B)    normed row b ready for layer l           (value l+1)
__device__ __forceinline__ void raise_abort(const DecParams &p);

__device__ __forceinline__ bool wait_ge(const DecParams &p, const unsigned *ctr, unsigned target, int *s_flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    const unsigned long long t0 = globaltimer_ns();
    uint32_t it = 0;
    while ((int)(ld_acquire_gpu(ctr) - target) < 0) {
      if ((++it & 31u) == 0) {
        if (ld_acquire_gpu(p.bar + 2)) { ok = 0; break; }
        if (globaltimer_ns() - t0 > p.timeout_ns) { raise_abort(p); ok = 0; break; }
      }
    }
    __threadfence();
    *s_flag = ok;
  }
  __syncthreads();
  return *s_flag != 0;
}

// Threads b < n wait for flags[b] >= target.
__device__ __forceinline__ bool wait_rows(const DecParams &p, const unsigned *flags, int n, unsigned target,
                                          int *s_flag) {
  if (threadIdx.x == 0) *s_flag = 1;
  __syncthreads();
  if ((int)threadIdx.x < n) {
    const unsigned long long t0 = globaltimer_ns();
    uint32_t it = 0;
    while ((int)(ld_acquire_gpu(flags + threadIdx.x) - target) < 0) {
      if ((++it & 31u) == 0 && (ld_acquire_gpu(p.bar + 2) || globaltimer_ns() - t0 > p.timeout_ns)) {
        raise_abort(p);
        *s_flag = 0;
        break;
      }
    }
    __threadfence();
  }
  __syncthreads();
  return *s_flag != 0;
}

// After the CTA's writes (callers end the tile with __syncthreads): publish.
__device__ __forceinline__ void signal_add(unsigned *ctr, unsigned n) {
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(ctr, n);
  }
}

__device__ __forceinline__ void raise_abort(const DecParams &p) {
  atomicExch(p.err, MTP_ERR_TIMEOUT);
  atomicExch(p.bar + 2, 1u);
}

// ----------------------------------------------------------------- staging and row tiles
// xs[b][0, klen) <- src[b][k0, k0 + klen) for b < B; rows B..NTP-1 zero.
__device__ __forceinline__ void stage_tokens(bf16 *xs, int xstride, const bf16 *src, int ld_src, int B, int NTP,
                                             int k0, int klen) {
  const int vpr = klen >> 3;
  for (int i = threadIdx.x; i < NTP * vpr; i += DT) {
    const int b = i / vpr, v = i - b * vpr;
    uint4 val = make_uint4(0u, 0u, 0u, 0u);
    if (b < B) val = __ldcg(reinterpret_cast<const uint4 *>(src + (size_t)b * ld_src + k0) + v);
    *reinterpret_cast<uint4 *>(xs + (size_t)b * xstride + 8 * v) = val;
  }
}

// 16 weight rows [r0, r0+16) of W (row-major, ld elements; rows >= nrows read as 0)
// times the staged tokens over k in [k0, k1) (xs column 0 = k0; k1 - k0 a multiple of 8,
// staged columns up to the next multiple of 32 zero, weights past k1 read as 0).  Warp w takes the
// 32-wide k blocks k0 + 32 w + 256 i.  Thread (g = lane/4, c = lane%4) loads 8
// consecutive k of rows g and g+8 as one 16-byte vector; the two m16n8k16 MMAs of a
// block use k {8c..8c+3} and {8c+4..8c+7}, and the token operand is loaded with the
// same k order, so each MMA sums over a permutation of its 16 k.
template <int NT>
__device__ __forceinline__ void tile_mma(const bf16 *__restrict__ W, int ld, int nrows, int r0, int k0, int k1,
                                         const bf16 *xs, int xstride, float (&acc)[NT][4]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, c = lane & 3;
  const bool va = r0 + g < nrows, vb = r0 + g + 8 < nrows;
  const bf16 *wa = W + (size_t)(va ? r0 + g : 0) * ld + 8 * c;
  const bf16 *wb = W + (size_t)(vb ? r0 + g + 8 : 0) * ld + 8 * c;
  const bf16 *xg = xs + (size_t)g * xstride + 8 * c;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
  constexpr int U = 8;
  for (int kb = k0 + 32 * warp; kb < k1; kb += 256 * U) {
    uint4 A[U], Bv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int k = kb + 256 * u;
      A[u] = (va && k + 8 * c < k1) ? ldg_stream(wa + k) : make_uint4(0u, 0u, 0u, 0u);
      Bv[u] = (vb && k + 8 * c < k1) ? ldg_stream(wb + k) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int k = kb + 256 * u;
      if (k < k1) {  // warp-uniform
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const uint4 X = *reinterpret_cast<const uint4 *>(xg + (size_t)nt * 8 * xstride + (k - k0));
          mma16816(acc[nt], A[u].x, Bv[u].x, A[u].y, Bv[u].y, X.x, X.y);
          mma16816(acc[nt], A[u].z, Bv[u].z, A[u].w, Bv[u].w, X.z, X.w);
        }
      }
    }
  }
}

// Sum the 8 warps' accumulators in warp order: red[w][row][tok]; afterwards thread t
// handles outputs o = t, t + 256, ... (row = o / NTP, tok = o % NTP) through f(row, tok, v).
template <int NT, typename F>
__device__ __forceinline__ void tile_finish(float (&acc)[NT][4], float *red, F f) {
  constexpr int NTP = NT * 8;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, c = lane & 3;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    float *rw = red + (size_t)warp * 16 * NTP;
    rw[g * NTP + nt * 8 + 2 * c] = acc[nt][0];
    rw[g * NTP + nt * 8 + 2 * c + 1] = acc[nt][1];
    rw[(g + 8) * NTP + nt * 8 + 2 * c] = acc[nt][2];
    rw[(g + 8) * NTP + nt * 8 + 2 * c + 1] = acc[nt][3];
  }
  __syncthreads();
  for (int o = threadIdx.x; o < 16 * NTP; o += DT) {
    float v = red[o];
#pragma unroll
    for (int w = 1; w < DW; ++w) v += red[(size_t)w * 16 * NTP + o];
    f(o / NTP, o % NTP, v);
  }
  __syncthreads();
}

// ----------------------------------------------------------------- one row's collective
// vals[q] holds element tid + q * DT of a row of `cols` fp32 values (the sum of this
// rank's partials).  Owner side: push the row's wire to every rank and raise its flag.
template <int VPT>
__device__ __forceinline__ void row_push(const DecParams &p, int site, int mode, int row, int rows, int cols,
                                         const float (&vals)[VPT], float *red32, uint32_t epoch) {
  const CommDev &d = p.cv;
  const int tid = threadIdx.x;
  float scale = 0.f;
  if (mode == MTP_RED_INT8TOK) {
    float m = 0.f;
#pragma unroll
    for (int q = 0; q < VPT; ++q)
      if (tid + q * DT < cols) m = fmaxf(m, fabsf(vals[q]));
    scale = q_scale(block_allreduce(m, red32, true));
  }
  const size_t half = (size_t)(epoch & 1u) * d.ws * d.slot_bytes[site];
  const size_t mine = d.off_recv[site] + half + (size_t)d.rank * d.slot_bytes[site];
  for (int k = 0; k < d.ws; ++k) {
    char *dst = d.peer[(d.rank + k) % d.ws] + mine;
    if (mode == MTP_RED_INT8TOK && tid == 0) reinterpret_cast<float *>(dst)[row] = scale;
#pragma unroll
    for (int q = 0; q < VPT; ++q) {
      const int c = tid + q * DT;
      if (c < cols) {
        if (mode == MTP_RED_FP32) reinterpret_cast<float *>(dst)[(size_t)row * cols + c] = vals[q];
        else if (mode == MTP_RED_FP16) reinterpret_cast<__half *>(dst)[(size_t)row * cols + c] = __float2half_rn(vals[q]);
        else reinterpret_cast<int8_t *>(dst + (size_t)4 * rows)[(size_t)row * cols + c] = (int8_t)q_one(vals[q], scale);
      }
    }
  }
  // barrier first, then one system fence per flag-writing thread (not per thread)
  __syncthreads();
  if (tid < d.ws) {
    __threadfence_system();
    st_release_sys(flag_ptr(d.peer[tid], d, site, 0, d.rank, row), epoch);
  }
}

// Wait for row `row` of every rank (bounded); false on timeout.
__device__ __forceinline__ bool row_wait(const DecParams &p, int site, int row, uint32_t epoch, int *s_flag) {
  const CommDev &d = p.cv;
  if (threadIdx.x == 0) *s_flag = 1;
  __syncthreads();
  if (threadIdx.x < d.ws) {
    const uint32_t *f = flag_ptr(d.peer[d.rank], d, site, 0, threadIdx.x, row);
    const unsigned long long t0 = globaltimer_ns();
    uint32_t it = 0;
    while ((int)(ld_acquire_sys(f) - epoch) < 0) {
      if ((++it & 63u) == 0 && globaltimer_ns() - t0 > d.timeout_ns) {
        atomicExch(reinterpret_cast<int *>(d.peer[d.rank] + d.off_status), MTP_ERR_TIMEOUT);
        *s_flag = 0;
        break;
      }
    }
    __threadfence();
  }
  __syncthreads();
  return *s_flag != 0;
}

// Rank-ordered reduction of element c of row `row` from this rank's receive slots.
__device__ __forceinline__ float row_reduce_elem(const DecParams &p, int site, int mode, int row, int rows, int cols,
                                                 int c, uint32_t epoch) {
  const CommDev &d = p.cv;
  const char *base = d.peer[d.rank] + d.off_recv[site] + (size_t)(epoch & 1u) * d.ws * d.slot_bytes[site];
  float a = 0.f;
  for (int k = 0; k < d.ws; ++k) {
    const char *sl = base + (size_t)k * d.slot_bytes[site];
    float v;
    if (mode == MTP_RED_FP32) {
      v = __ldcg(reinterpret_cast<const float *>(sl) + (size_t)row * cols + c);
    } else if (mode == MTP_RED_FP16) {
      v = __half2float(__ushort_as_half(__ldcg(reinterpret_cast<const unsigned short *>(sl) + (size_t)row * cols + c)));
    } else {
      const float s = __ldcg(reinterpret_cast<const float *>(sl) + row);
      v = __fmul_rn((float)*(const volatile int8_t *)(sl + (size_t)4 * rows + (size_t)row * cols + c), s);
    }
    a = __fadd_rn(a, v);
  }
  if (mode == MTP_RED_FP16) a = __half2float(__float2half_rn(a));
  return bf(a);
}

// World size 1: the wire format's round trip of one row held as vals (same layout as row_push).
template <int VPT>
__device__ __forceinline__ void row_roundtrip(int mode, int cols, float (&vals)[VPT], float *red32) {
  const int tid = threadIdx.x;
  float scale = 0.f;
  if (mode == MTP_RED_INT8TOK) {
    float m = 0.f;
#pragma unroll
    for (int q = 0; q < VPT; ++q)
      if (tid + q * DT < cols) m = fmaxf(m, fabsf(vals[q]));
    scale = q_scale(block_allreduce(m, red32, true));
  }
#pragma unroll
  for (int q = 0; q < VPT; ++q) {
    float v = vals[q];
    if (mode == MTP_RED_FP16) v = __half2float(__float2half_rn(v));
    else if (mode == MTP_RED_INT8TOK) v = __fadd_rn(0.f, __fmul_rn((float)q_one(v, scale), scale));
    vals[q] = bf(v);
  }
}

// ----------------------------------------------------------------- L2 prefetch of each phase's inputs
// Latency-critical small reads (parameters, cache state) are requested before the
// large weight streams, so they do not queue behind them in HBM.
__device__ __forceinline__ void prefetch_p1(const DecParams &p, const DecLayer &Ly, const DecCache &Cc, int lane) {
  const int U = (2 * p.Es + 15) / 16;
  for (int u = blockIdx.x; u < U; u += gridDim.x) {
    const int r0 = 16 * u;
    if (r0 < p.Es) {
      if (lane == 0) prefetch_l2(Ly.conv_w + (size_t)r0 * DK, 16 * DK * 2);
      if (lane == 1 && Ly.conv_b) prefetch_l2(Ly.conv_b + r0, 32);
      for (int b = lane; b < p.B; b += 32) prefetch_l2(Cc.conv + ((size_t)b * p.Es + r0) * (DK - 1), 16 * (DK - 1) * 2);
    }
    if (lane == 2 && Ly.in_b) prefetch_l2(Ly.in_b + r0, 32);
  }
  for (int u = blockIdx.x; u < U; u += gridDim.x) {
    const int r0 = 16 * u, nr = min(16, 2 * p.Es - r0);
    prefetch_range(Ly.in_w + (size_t)r0 * p.D, (size_t)nr * p.D * 2, lane);
  }
}

__device__ __forceinline__ void prefetch_p2_to_p6(const DecParams &p, const DecLayer &Ly, const DecCache &Cc,
                                                  const bf16 *next_norm, int lane) {
  // P4: per 16-channel tile its SSM state rows, dt_proj rows, A_log, bias, D
  for (int u = blockIdx.x; u < p.Es / 16; u += gridDim.x) {
    const int c0 = 16 * u;
    for (int b = lane; b < p.B; b += 32) prefetch_l2(Cc.ssm + ((size_t)b * p.Es + c0) * DN, 16 * DN * 4);
    if (lane == 0) prefetch_l2(Ly.A_log + (size_t)c0 * DN, 16 * DN * 2);
    if (lane == 1) prefetch_l2(Ly.dt_b + c0, 32);
    if (lane == 2) prefetch_l2(Ly.Dp + c0, 32);
    if (lane == 3) prefetch_l2(Ly.dt_w + (size_t)c0 * p.R, (uint32_t)(16 * p.R * 2));
  }
  // P6: the owner's norm weight and out_proj bias
  if (blockIdx.x < p.B) {
    prefetch_range(next_norm, (size_t)p.D * 2, lane);
    if (Ly.out_b) prefetch_range(Ly.out_b, (size_t)p.D * 2, lane);
  }
  // P2: x_proj tiles
  const int RTx = (p.NX + 15) / 16;
  for (int u = blockIdx.x; u < RTx * p.KCx; u += gridDim.x) {
    const int rt = u % RTx, kc = u / RTx, k0 = kc * p.chunk_x, k1 = min(p.Es, k0 + p.chunk_x);
    for (int r = 16 * rt + lane; r < min(p.NX, 16 * rt + 16); r += 32)
      prefetch_l2(Ly.x_w + (size_t)r * p.Es + k0, (uint32_t)(k1 - k0) * 2);
  }
  // P5: out_proj tiles
  const int RTo = (p.D + 15) / 16;
  for (int u = blockIdx.x; u < RTo * p.KCo; u += gridDim.x) {
    const int rt = u % RTo, kc = u / RTo, k0 = kc * p.chunk_o, k1 = min(p.Es, k0 + p.chunk_o);
    const int r0 = 16 * rt, nr = min(16, p.D - r0);
    if (k0 == 0 && k1 == p.Es) {
      prefetch_range(Ly.out_w + (size_t)r0 * p.Es, (size_t)nr * p.Es * 2, lane);
    } else {
      for (int r = r0 + lane; r < r0 + nr; r += 32) prefetch_l2(Ly.out_w + (size_t)r * p.Es + k0, (uint32_t)(k1 - k0) * 2);
    }
  }
}

// True (for the whole CTA) once some wait of the launch has given up.
__device__ __forceinline__ bool bar_aborted(const DecParams &p) {
  __shared__ int s_ab;
  __syncthreads();
  if (threadIdx.x == 0) s_ab = ld_acquire_gpu(p.bar + 2) != 0u;
  __syncthreads();
  return s_ab != 0;
}

__device__ __forceinline__ void st_release_gpu(unsigned *p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// ----------------------------------------------------------------- the kernel
template <int NT, int VPT_D>
__global__ void __launch_bounds__(DT, 1) decode_kernel(DecParams p) {
  extern __shared__ __align__(16) unsigned char dsm[];
  __shared__ float red32[32];
  __shared__ int s_flag;
  __shared__ uint32_t s_epoch[3];
  constexpr int NTP = NT * 8;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, B = p.B, D = p.D, Es = p.Es, R = p.R, NX = p.NX;
  // shared memory: token staging | warp partial sums | B|C rows | dt of a tile | A of a tile
  bf16 *xs = reinterpret_cast<bf16 *>(dsm);
  float *red = reinterpret_cast<float *>(dsm + (size_t)NTP * p.xstride * 2);
  float *bcs = red + DW * 16 * NTP;  // [B][2N]
  float *dts = bcs + NTP * 2 * DN;   // [16][NTP]
  float *a2s = dts + 16 * NTP;       // [16][N]
  if (p.trace && tid == 0 && blockIdx.x == 0) p.trace[0] = globaltimer_ns();
  auto stamp = [&](int k) {
    if (p.trace && tid == 0 && blockIdx.x == 0) p.trace[k] = globaltimer_ns();
  };
  unsigned *c1 = p.cnt, *cz = p.cnt + p.KCx, *c2 = cz + 1, *c4 = c2 + 1, *c5 = c4 + p.KCo, *nflag = c5 + 1;
  if (tid == 0) {
    s_epoch[0] = p.has_comm ? *reinterpret_cast<volatile uint32_t *>(p.cv.peer[p.cv.rank] + p.cv.off_epoch) : 0u;
    s_epoch[1] = p.has_comm ? *reinterpret_cast<volatile uint32_t *>(p.cv.peer[p.cv.rank] + p.cv.off_epoch + 4) : 0u;
    s_epoch[2] = *reinterpret_cast<volatile uint32_t *>(p.lepoch);
  }
  __syncthreads();
  uint32_t ep_x = s_epoch[0], ep_o = s_epoch[1];
  const uint32_t lep0 = s_epoch[2];
  const int RTx = (NX + 15) / 16, RTo = (D + 15) / 16, U1 = (2 * Es + 15) / 16, U4 = Es / 16;
  const int Rp = (R + 31) & ~31;  // dt_low staged width (zero padded)
  // states per thread in the step: 16 * B * SPLIT <= 256 threads where possible
  const int SPLIT = B >= 16 ? 1 : B >= 8 ? 2 : B >= 4 ? 4 : B >= 2 ? 8 : 16;
  const int NS = DN / SPLIT;

  // ---------------- P0: embedding row, first RMSNorm (owner CTA per token; the owner keeps
  // its token's fp32 residual stream in registers for the whole step)
  float resid[VPT_D];
  if (p.prefetch && warp == 0) prefetch_p1(p, p.layers[0], p.cache[0], lane);
  if (blockIdx.x < B) {
    const int b = blockIdx.x;
    const bf16 *er = p.emb + (size_t)p.ids[b] * D;
    const bf16 *nw = p.layers[0].norm_w;
    float ss = 0.f;
#pragma unroll
    for (int q = 0; q < VPT_D; ++q) {
      const int c = tid + q * DT;
      resid[q] = c < D ? ldbf(er + c) : 0.f;
      ss += resid[q] * resid[q];
    }
    const float rs = rsqrtf(block_allreduce(ss, red32, false) / (float)D + p.eps);
#pragma unroll
    for (int q = 0; q < VPT_D; ++q) {
      const int c = tid + q * DT;
      if (c < D) p.normed[(size_t)b * D + c] = __float2bfloat16_rn(ldbf(nw + c) * (resid[q] * rs));
    }
    __syncthreads();
    if (tid == 0) {
      __threadfence();
      st_release_gpu(nflag + b, 1u);
    }
  }
  stamp(1);

  for (int l = 0; l < p.n_layer; ++l) {
    const DecLayer Ly = p.layers[l];
    const DecCache Cc = p.cache[l];
    const bf16 *next_norm = l + 1 < p.n_layer ? p.layers[l + 1].norm_w : p.norm_f;
    // ---------------- P1: in_proj + conv
    if (p.prefetch && warp == 0) prefetch_p2_to_p6(p, Ly, Cc, next_norm, lane);
    if (blockIdx.x < U1) {
      if (!wait_rows(p, nflag, B, (unsigned)l + 1u, &s_flag)) return;  // every token's normed row
      stage_tokens(xs, p.xstride, p.normed, D, B, NTP, 0, D);
    }
    __syncthreads();
    for (int u = blockIdx.x; u < U1; u += G) {
      float acc[NT][4];
      const int r0 = 16 * u;
      tile_mma<NT>(Ly.in_w, D, 2 * Es, r0, 0, D, xs, p.xstride, acc);
      tile_finish<NT>(acc, red, [&](int row, int tok, float v) {
        const int n = r0 + row;
        if (tok >= B || n >= 2 * Es) return;
        if (Ly.in_b) v += ldbf(Ly.in_b + n);
        const float xz = bf(v);
        if (n < Es) {
          bf16 *hs = Cc.conv + ((size_t)tok * Es + n) * (DK - 1);
          const bf16 *w = Ly.conv_w + (size_t)n * DK;
          float h[DK - 1];
#pragma unroll
          for (int j = 0; j < DK - 1; ++j) h[j] = ldbf(hs + j);
          float a = Ly.conv_b ? ldbf(Ly.conv_b + n) : 0.f;
#pragma unroll
          for (int j = 0; j < DK - 1; ++j) a = fmaf(ldbf(w + j), h[j], a);
          a = fmaf(ldbf(w + DK - 1), xz, a);
#pragma unroll
          for (int j = 0; j < DK - 2; ++j) hs[j] = __float2bfloat16_rn(h[j + 1]);
          hs[DK - 2] = __float2bfloat16_rn(xz);
          const float xc = silu_f(a);
          p.xcf[(size_t)tok * Es + n] = xc;
          p.xcT[(size_t)tok * Es + n] = __float2bfloat16_rn(xc);
        } else {
          p.zT[(size_t)tok * Es + (n - Es)] = __float2bfloat16_rn(xz);
        }
      });
      signal_add(16 * u < Es ? c1 + (16 * u) / p.chunk_x : cz, 1u);
    }
    stamp(2 + 5 * l);
    // ---------------- P2: x_proj partials
    if (p.prefetch && warp == 0 && l + 1 < p.n_layer) prefetch_p1(p, p.layers[l + 1], p.cache[l + 1], lane);
    {
      int staged = -1;
      for (int u = blockIdx.x; u < RTx * p.KCx; u += G) {
        const int rt = u % RTx, kc = u / RTx, k0 = kc * p.chunk_x, k1 = min(Es, k0 + p.chunk_x);
        if (kc != staged) {  // this K chunk's in_proj x tiles
          if (!wait_ge(p, c1 + kc, (unsigned)(l + 1) * (unsigned)((k1 - k0) / 16), &s_flag)) return;
          stage_tokens(xs, p.xstride, p.xcT, Es, B, NTP, k0, k1 - k0);
          __syncthreads();
          staged = kc;
        }
        float acc[NT][4];
        tile_mma<NT>(Ly.x_w, Es, NX, 16 * rt, k0, k1, xs, p.xstride, acc);
        tile_finish<NT>(acc, red, [&](int row, int tok, float v) {
          const int n = 16 * rt + row;
          if (tok < B && n < NX) p.pxp[((size_t)kc * B + tok) * NX + n] = v;
        });
        signal_add(c2, 1u);
      }
    }
    stamp(3 + 5 * l);
    // ---------------- P3: owner CTA b reduces row b of x_proj (AllReduce #1) and publishes it
    const uint32_t lep = lep0 + (uint32_t)l + 1u;
    if (p.has_comm) ++ep_x;
    if (blockIdx.x < B) {
      const int b = blockIdx.x;
      if (!wait_ge(p, c2, (unsigned)(l + 1) * (unsigned)(RTx * p.KCx), &s_flag)) return;  // all x_proj units
      float v[2];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int c = tid + q * DT;
        float a = 0.f;
        if (c < NX)
          for (int kc = 0; kc < p.KCx; ++kc) a += __ldcg(p.pxp + ((size_t)kc * B + b) * NX + c);
        v[q] = a;
      }
      bool ok = true;
      if (p.has_comm) {
        row_push<2>(p, 0, Ly.mode_x, b, B, NX, v, red32, ep_x);
        ok = row_wait(p, 0, b, ep_x, &s_flag);
        if (ok) {
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const int c = tid + q * DT;
            if (c < NX) v[q] = row_reduce_elem(p, 0, Ly.mode_x, b, B, NX, c, ep_x);
          }
        } else {
          raise_abort(p);
        }
      } else {
        row_roundtrip<2>(Ly.mode_x, NX, v, red32);
      }
      if (ok) {
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int c = tid + q * DT;
          if (c < NX) p.xd[(size_t)b * NX + c] = v[q];
        }
        __syncthreads();
        if (tid == 0) {
          __threadfence();
          st_release_gpu(p.lflags + b, lep);
        }
      }
    }
    // ---------------- P4: the step, 16-channel tiles; dt_proj on the tensor cores
    if (blockIdx.x < U4) {
      if (tid == 0) s_flag = 1;
      __syncthreads();
      if (tid < B) {  // wait for every token's reduced row
        const unsigned long long t0 = globaltimer_ns();
        uint32_t it = 0;
        while ((int)(ld_acquire_gpu(p.lflags + tid) - lep) < 0) {
          if ((++it & 31u) == 0 && (ld_acquire_gpu(p.bar + 2) || globaltimer_ns() - t0 > p.timeout_ns)) {
            raise_abort(p);
            s_flag = 0;
            break;
          }
        }
      }
      __syncthreads();
      if (s_flag && !wait_ge(p, cz, (unsigned)(l + 1) * (unsigned)(Es / 16), &s_flag)) return;  // z tiles
      if (s_flag) {
        // dt_low (bf16 values) as MMA tokens, B|C rows as fp32
        for (int i = tid; i < NTP * Rp; i += DT) {
          const int b = i / Rp, r = i - b * Rp;
          xs[(size_t)b * p.xstride + r] = __float2bfloat16_rn(b < B && r < R ? __ldcg(p.xd + (size_t)b * NX + r) : 0.f);
        }
        for (int i = tid; i < B * 2 * DN; i += DT) {
          const int b = i / (2 * DN), j = i - b * (2 * DN);
          bcs[i] = __ldcg(p.xd + (size_t)b * NX + R + j);
        }
        __syncthreads();
        for (int u = blockIdx.x; u < U4; u += G) {
          const int c0 = 16 * u;
          a2s[tid] = -expf(ldbf(Ly.A_log + (size_t)c0 * DN + tid)) * 1.4426950408889634f;  // 16 x 16 = DT values
          float acc[NT][4];
          tile_mma<NT>(Ly.dt_w, R, Es, c0, 0, R, xs, p.xstride, acc);
          tile_finish<NT>(acc, red, [&](int row, int tok, float v) {
            dts[row * NTP + tok] = tok < B ? softplus_f(v + ldbf(Ly.dt_b + c0 + row)) : 0.f;
          });
          const int total = 16 * B * SPLIT;
          for (int base = 0; base < total; base += DT) {
            const int idx = base + tid;
            const bool act = idx < total;
            const int pair = act ? idx / SPLIT : 0, part = idx - (idx / SPLIT) * SPLIT;
            const int row = pair & 15, tok = pair >> 4, c = c0 + row;
            float yp = 0.f, xc = 0.f;
            if (act) {
              const float dt = dts[row * NTP + tok];
              xc = __ldcg(p.xcf + (size_t)tok * Es + c);
              const float dtx = dt * xc;
              float *st = Cc.ssm + ((size_t)tok * Es + c) * DN + part * NS;
              const float *bb = bcs + tok * 2 * DN + part * NS;
              const float *a2 = a2s + row * DN + part * NS;
              for (int n = 0; n < NS; ++n) {
                float dA;
                asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(dA) : "f"(dt * a2[n]));
                const float h = fmaf(dA, st[n], bb[n] * dtx);
                st[n] = h;
                yp = fmaf(bb[DN + n], h, yp);
              }
            }
            for (int o = 1; o < SPLIT; o <<= 1) yp += __shfl_xor_sync(0xffffffffu, yp, o);
            if (act && part == 0) {
              const float zv = ldcg_bf(p.zT + (size_t)tok * Es + c);
              p.yT[(size_t)tok * Es + c] = __float2bfloat16_rn(fmaf(ldbf(Ly.Dp + c), xc, yp) * silu_f(zv));
            }
          }
          __syncthreads();
          signal_add(c4 + c0 / p.chunk_o, 1u);
        }
      }
    }
    if (bar_aborted(p)) return;
    stamp(4 + 5 * l);
    // ---------------- P5: out_proj partials
    {
      int staged = -1;
      for (int u = blockIdx.x; u < RTo * p.KCo; u += G) {
        const int rt = u % RTo, kc = u / RTo, k0 = kc * p.chunk_o, k1 = min(Es, k0 + p.chunk_o);
        if (kc != staged) {  // this K chunk's step tiles
          if (!wait_ge(p, c4 + kc, (unsigned)(l + 1) * (unsigned)((k1 - k0) / 16), &s_flag)) return;
          stage_tokens(xs, p.xstride, p.yT, Es, B, NTP, k0, k1 - k0);
          __syncthreads();
          staged = kc;
        }
        float acc[NT][4];
        tile_mma<NT>(Ly.out_w, Es, D, 16 * rt, k0, k1, xs, p.xstride, acc);
        tile_finish<NT>(acc, red, [&](int row, int tok, float v) {
          const int n = 16 * rt + row;
          if (tok < B && n < D) p.pop[((size_t)kc * B + tok) * D + n] = v;
        });
        signal_add(c5, 1u);
      }
    }
    stamp(5 + 5 * l);
    // ---------------- P6: AllReduce #2 + bias + residual + next RMSNorm (owner CTA per token)
    if (p.has_comm) ++ep_o;
    if (blockIdx.x < B) {
      const int b = blockIdx.x;
      if (!wait_ge(p, c5, (unsigned)(l + 1) * (unsigned)(RTo * p.KCo), &s_flag)) return;  // all out_proj units
      float v[VPT_D];
#pragma unroll
      for (int q = 0; q < VPT_D; ++q) {
        const int c = tid + q * DT;
        float a = 0.f;
        if (c < D)
          for (int kc = 0; kc < p.KCo; ++kc) a += __ldcg(p.pop + ((size_t)kc * B + b) * D + c);
        v[q] = a;
      }
      bool ok = true;
      if (p.has_comm) {
        row_push<VPT_D>(p, 1, Ly.mode_out, b, B, D, v, red32, ep_o);
        ok = row_wait(p, 1, b, ep_o, &s_flag);
        if (ok) {
#pragma unroll
          for (int q = 0; q < VPT_D; ++q) {
            const int c = tid + q * DT;
            if (c < D) v[q] = row_reduce_elem(p, 1, Ly.mode_out, b, B, D, c, ep_o);
          }
        } else {
          raise_abort(p);
        }
      } else {
        row_roundtrip<VPT_D>(Ly.mode_out, D, v, red32);
      }
      if (ok) {
        float ss = 0.f;
#pragma unroll
        for (int q = 0; q < VPT_D; ++q) {
          const int c = tid + q * DT;
          if (c < D) {
            const float o = Ly.out_b ? v[q] + ldbf(Ly.out_b + c) : v[q];
            resid[q] = resid[q] + o;
            ss += resid[q] * resid[q];
          }
        }
        const float rs = rsqrtf(block_allreduce(ss, red32, false) / (float)D + p.eps);
#pragma unroll
        for (int q = 0; q < VPT_D; ++q) {
          const int c = tid + q * DT;
          if (c < D) p.normed[(size_t)b * D + c] = __float2bfloat16_rn(ldbf(next_norm + c) * (resid[q] * rs));
        }
        __syncthreads();
        if (tid == 0) {
          __threadfence();
          st_release_gpu(nflag + b, (unsigned)l + 2u);
        }
      }
    }
    if (bar_aborted(p)) return;
    stamp(6 + 5 * l);
  }
  // exit: publish the epochs; the last CTA out resets the barrier counters
  if (tid == 0) {
    if (blockIdx.x == 0) {
      if (p.has_comm) {
        *reinterpret_cast<volatile uint32_t *>(p.cv.peer[p.cv.rank] + p.cv.off_epoch) = ep_x;
        *reinterpret_cast<volatile uint32_t *>(p.cv.peer[p.cv.rank] + p.cv.off_epoch + 4) = ep_o;
      }
      *reinterpret_cast<volatile uint32_t *>(p.lepoch) = lep0 + (uint32_t)p.n_layer;
    }
    __threadfence();
    if (atomicAdd(p.bar + 1, 1u) == (unsigned)G - 1u) {  // every CTA is done: reset for the next launch
      for (int i = 0; i < p.ncnt; ++i) p.cnt[i] = 0u;
      p.bar[1] = 0u;
      __threadfence();
    }
  }
}

template <int NT, int V>
static cudaError_t launch_decode(const DecParams &p, int G, size_t smem, cudaStream_t s) {
  auto kern = decode_kernel<NT, V>;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(DT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int NT>
static cudaError_t launch_decode_v(const DecParams &p, int G, size_t smem, cudaStream_t s) {
  if (p.D <= 4 * DT) return launch_decode<NT, 4>(p, G, smem, s);
  if (p.D <= 8 * DT) return launch_decode<NT, 8>(p, G, smem, s);
  return launch_decode<NT, 12>(p, G, smem, s);
}

}  // namespace mtp

using namespace mtp;

struct mtp_decode_plan {
  DecParams p{};  // B, ids, cache, normed filled per call
  DecLayer *d_layers = nullptr;
  void *scratch = nullptr;
  unsigned *bar = nullptr;
  int max_batch = 0, grid = 0, n_layer = 0;
  int D = 0, Es = 0, R = 0, NX = 0;
  int comm_max_rows = 0;
  unsigned long long *trace_buf = nullptr;
  int n_trace = 0;
  size_t cnt_bytes = 0;
  size_t lflags_bytes = 0;  // per-row publication flags + local epoch
};

struct mtp_decode_cache {
  DecCache *d_cache = nullptr;
  int batch = 0, n_layer = 0;
};

static size_t decode_smem(int B, int xstride) {
  const int NTP = ((B + 7) / 8) * 8;
  return (size_t)NTP * xstride * 2 + ((size_t)DW * 16 * NTP + (size_t)NTP * 2 * DN + 16 * (size_t)NTP + 16 * DN) * 4;
}

extern "C" {

int mtp_decode_plan_create(const mtp_decode_layer *layers, int n_layer, const void *norm_f, const void *embedding,
                           int d_model, int d_inner, int d_state, int dt_rank, int d_conv, float eps, int max_batch,
                           int dtype, mtp_comm *comm, mtp_decode_plan **out) {
  MTP_REQUIRE(out && layers && norm_f && embedding && n_layer > 0, "bad arguments");
  MTP_REQUIRE(aligned16(norm_f) && aligned16(embedding), "norm_f and the embedding must be 16-byte aligned");
  MTP_REQUIRE(dtype == MTP_BF16, "the persistent decode kernel runs bf16 models");
  MTP_REQUIRE(d_state == DN && d_conv == DK, "the persistent decode kernel needs d_state 16 and d_conv 4");
  MTP_REQUIRE(d_model % 32 == 0 && d_model <= 12 * DT, "d_model must be a multiple of 32 and at most 3072");
  MTP_REQUIRE(d_inner % 32 == 0 && d_inner > 0, "d_inner (per rank) must be a multiple of 32");
  MTP_REQUIRE(dt_rank % 8 == 0 && dt_rank > 0, "dt_rank must be a multiple of 8");
  const int NX = dt_rank + 2 * d_state;
  MTP_REQUIRE(NX <= 2 * DT, "dt_rank + 2 d_state must be at most 512");
  MTP_REQUIRE(max_batch >= 1 && max_batch <= 32, "max_batch must be in [1, 32]");
  MTP_REQUIRE(dt_rank <= d_model, "dt_rank must not exceed d_model");
  const bool has_comm = comm && comm->d.ws > 1;
  if (has_comm) {
    MTP_REQUIRE(comm->opened, "comm context peers not opened");
    MTP_REQUIRE(max_batch <= comm->max_rows && max_batch <= G_MAX, "max_batch exceeds the comm context's rows");
    MTP_REQUIRE(comm->cols[0] >= NX && comm->cols[1] >= d_model, "comm context site widths too small");
  }
  for (int l = 0; l < n_layer; ++l) {
    const mtp_decode_layer &L = layers[l];
    MTP_REQUIRE(L.norm_w && L.in_w && L.conv_w && L.x_w && L.dt_w && L.dt_b && L.A_log && L.Dp && L.out_w,
                "missing layer weight");
    // every pointer the kernel reads with vector loads or L2 bulk prefetches: 16-byte aligned
    for (const void *q : {L.norm_w, L.in_w, L.in_b, L.conv_w, L.conv_b, L.x_w, L.dt_w, L.dt_b, L.A_log, L.Dp, L.out_w,
                          L.out_b})
      MTP_REQUIRE(!q || aligned16(q), "layer weights must be 16-byte aligned");
    for (int m : {L.mode_x, L.mode_out})
      MTP_REQUIRE(m == MTP_RED_FP32 || m == MTP_RED_FP16 || m == MTP_RED_INT8TOK, "unknown reduction mode");
  }
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = num_sms();
  MTP_REQUIRE(max_batch <= sms, "max_batch exceeds the number of SMs (one owner CTA per token)");
  mtp_decode_plan *P = new mtp_decode_plan();
  P->max_batch = max_batch;
  P->n_layer = n_layer;
  P->D = d_model;
  P->Es = d_inner;
  P->R = dt_rank;
  P->NX = NX;
  DecParams &p = P->p;
  p.n_layer = n_layer;
  p.norm_f = (const bf16 *)norm_f;
  p.emb = (const bf16 *)embedding;
  p.D = d_model;
  p.Es = d_inner;
  p.R = dt_rank;
  p.NX = NX;
  p.eps = eps;
  // split of the x_proj and out_proj K (= d_inner) over CTAs: about one unit per SM
  const int RTx = (NX + 15) / 16, RTo = (d_model + 15) / 16;
  int kcx = sms / RTx;
  if (kcx < 1) kcx = 1;
  if (kcx > d_inner / 256) kcx = d_inner / 256 > 0 ? d_inner / 256 : 1;
  // the staged token rows are at most d_model wide: K chunks never exceed it
  p.chunk_x = ceil_div(ceil_div(d_inner, kcx), 32) * 32;
  if (p.chunk_x > d_model) p.chunk_x = d_model;
  p.KCx = ceil_div(d_inner, p.chunk_x);
  int kco = sms / RTo;
  if (kco < 1) kco = 1;
  if (kco > d_inner / 256) kco = d_inner / 256 > 0 ? d_inner / 256 : 1;
  p.chunk_o = ceil_div(ceil_div(d_inner, kco), 32) * 32;
  if (p.chunk_o > d_model) p.chunk_o = d_model;
  p.KCo = ceil_div(d_inner, p.chunk_o);
  p.xstride = d_model + XPAD;
  const size_t smem = decode_smem(max_batch, p.xstride);
  if (smem > 200 * 1024) {
    delete P;
    return fail(MTP_ERR_UNSUPPORTED, "decode plan needs more than 200 KB of shared memory (lower max_batch)");
  }
  p.has_comm = has_comm ? 1 : 0;
  {
    const char *e = getenv("MTP_DECODE_PREFETCH");
    p.prefetch = (e && e[0] == '0') ? 0 : 1;
  }
  if (has_comm) {
    p.cv = comm->d;
    P->comm_max_rows = comm->max_rows;
  }
  p.timeout_ns = has_comm ? comm->d.timeout_ns : 10ull * 1000000000ull;
  // device layer table and scratch
  std::vector<DecLayer> host(n_layer);
  for (int l = 0; l < n_layer; ++l) {
    const mtp_decode_layer &L = layers[l];
    host[l] = DecLayer{(const bf16 *)L.norm_w, (const bf16 *)L.in_w, (const bf16 *)L.in_b, (const bf16 *)L.conv_w,
                       (const bf16 *)L.conv_b, (const bf16 *)L.x_w, (const bf16 *)L.dt_w, (const bf16 *)L.dt_b,
                       (const bf16 *)L.A_log, (const bf16 *)L.Dp, (const bf16 *)L.out_w, (const bf16 *)L.out_b,
                       L.mode_x, L.mode_out};
  }
  const size_t MB = max_batch;
  auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
  size_t off = 0;
  const size_t o_layers = off; off = al(off + sizeof(DecLayer) * n_layer);
  const size_t o_xcf = off; off = al(off + MB * d_inner * 4);
  const size_t o_xcT = off; off = al(off + MB * d_inner * 2);
  const size_t o_zT = off; off = al(off + MB * d_inner * 2);
  const size_t o_yT = off; off = al(off + MB * d_inner * 2);
  const size_t o_pxp = off; off = al(off + (size_t)p.KCx * MB * NX * 4);
  const size_t o_pop = off; off = al(off + (size_t)p.KCo * MB * d_model * 4);
  const size_t o_xd = off; off = al(off + MB * NX * 4);
  const size_t o_lflags = off; off = al(off + MB * 4 + 4);
  const size_t o_bar = off; off = al(off + 64);
  const int ncnt = p.KCx + p.KCo + 3 + max_batch;
  const size_t o_cnt = off; off = al(off + sizeof(unsigned) * ncnt);
  const size_t n_trace = (size_t)(2 + 5 * n_layer);
  const size_t o_trace = off; off = al(off + n_trace * 8);
  char *base = nullptr;
  if (cudaMalloc(&base, off) != cudaSuccess) {
    delete P;
    return fail(MTP_ERR_CUDA, "cudaMalloc of the decode plan failed");
  }
  P->scratch = base;
  cudaMemset(base, 0, off);
  cudaMemcpy(base + o_layers, host.data(), sizeof(DecLayer) * n_layer, cudaMemcpyHostToDevice);
  P->d_layers = reinterpret_cast<DecLayer *>(base + o_layers);
  p.layers = P->d_layers;
  p.xd = reinterpret_cast<float *>(base + o_xd);
  p.lflags = reinterpret_cast<unsigned *>(base + o_lflags);
  p.lepoch = reinterpret_cast<unsigned *>(base + o_lflags + MB * 4);
  p.xcf = reinterpret_cast<float *>(base + o_xcf);
  p.xcT = reinterpret_cast<bf16 *>(base + o_xcT);
  p.zT = reinterpret_cast<bf16 *>(base + o_zT);
  p.yT = reinterpret_cast<bf16 *>(base + o_yT);
  p.pxp = reinterpret_cast<float *>(base + o_pxp);
  p.pop = reinterpret_cast<float *>(base + o_pop);
  P->bar = reinterpret_cast<unsigned *>(base + o_bar);
  p.bar = P->bar;
  p.err = reinterpret_cast<int *>(base + o_bar + 16);
  p.cnt = reinterpret_cast<unsigned *>(base + o_cnt);
  p.ncnt = ncnt;
  P->cnt_bytes = sizeof(unsigned) * ncnt;
  P->lflags_bytes = (size_t)MB * 4 + 4;
  P->trace_buf = reinterpret_cast<unsigned long long *>(base + o_trace);
  P->n_trace = (int)n_trace;
  p.trace = nullptr;
  // one CTA per SM, provided the occupancy calculator agrees
  int per_sm = 0;
  cudaFuncSetAttribute(decode_kernel<4, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_kernel<4, 8>, DT, smem);
  if (cudaGetLastError() != cudaSuccess || per_sm < 1) {
    cudaFree(base);
    delete P;
    return fail(MTP_ERR_CUDA, "persistent decode kernel does not fit one CTA per SM");
  }
  P->grid = sms;
  *out = P;
  return MTP_OK;
}

int mtp_decode_bind_cache(mtp_decode_plan *P, void *const *conv_state, float *const *ssm_state, int batch,
                          mtp_decode_cache **out) {
  MTP_REQUIRE(P && conv_state && ssm_state && out, "bad arguments");
  MTP_REQUIRE(batch >= 1 && batch <= P->max_batch, "batch exceeds the plan's max_batch");
  std::vector<DecCache> host(P->n_layer);
  for (int l = 0; l < P->n_layer; ++l) {
    MTP_REQUIRE(conv_state[l] && ssm_state[l] && aligned16(conv_state[l]) && aligned16(ssm_state[l]),
                "cache tensors must be non-null and 16-byte aligned");
    host[l] = DecCache{(bf16 *)conv_state[l], ssm_state[l]};
  }
  mtp_decode_cache *c = new mtp_decode_cache();
  if (cudaMalloc(&c->d_cache, sizeof(DecCache) * P->n_layer) != cudaSuccess) {
    delete c;
    return fail(MTP_ERR_CUDA, "cudaMalloc of the cache table failed");
  }
  cudaMemcpy(c->d_cache, host.data(), sizeof(DecCache) * P->n_layer, cudaMemcpyHostToDevice);
  c->batch = batch;
  c->n_layer = P->n_layer;
  *out = c;
  return MTP_OK;
}

int mtp_decode_step(mtp_decode_plan *P, mtp_decode_cache *c, const int64_t *ids, void *normed, void *stream) {
  MTP_REQUIRE(P && c && ids && normed, "bad arguments");
  MTP_REQUIRE(c->n_layer == P->n_layer, "cache binding belongs to another plan");
  MTP_REQUIRE(aligned16(normed), "normed must be 16-byte aligned");
  DecParams p = P->p;
  p.B = c->batch;
  p.cache = c->d_cache;
  p.ids = ids;
  p.normed = (bf16 *)normed;
  const int NT = (p.B + 7) / 8;
  const size_t smem = decode_smem(p.B, p.xstride);
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e;
  switch (NT) {
    case 1: e = launch_decode_v<1>(p, P->grid, smem, s); break;
    case 2: e = launch_decode_v<2>(p, P->grid, smem, s); break;
    case 3: e = launch_decode_v<3>(p, P->grid, smem, s); break;
    default: e = launch_decode_v<4>(p, P->grid, smem, s); break;
  }
  if (e != cudaSuccess) return fail(MTP_ERR_CUDA, std::string("decode launch: ") + cudaGetErrorString(e));
  return check_launch("decode");
}

int mtp_decode_status(mtp_decode_plan *P, int *status) {
  MTP_REQUIRE(P && status, "bad arguments");
  if (cudaMemcpy(status, P->p.err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return fail(MTP_ERR_CUDA, "reading the decode status failed");
  return MTP_OK;
}

int mtp_decode_reset(mtp_decode_plan *P) {
  MTP_REQUIRE(P, "bad arguments");
  // an aborted step leaves row flags ahead of the local epoch: clear both with the counters
  if (cudaMemset(P->bar, 0, 64) != cudaSuccess || cudaMemset(P->p.cnt, 0, P->cnt_bytes) != cudaSuccess ||
      cudaMemset(P->p.lflags, 0, P->lflags_bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess)
    return fail(MTP_ERR_CUDA, "reset of the decode counters failed");
  return MTP_OK;
}

int mtp_decode_set_trace(mtp_decode_plan *P, int on) {
  MTP_REQUIRE(P, "bad arguments");
  P->p.trace = on ? P->trace_buf : nullptr;
  return MTP_OK;
}

int mtp_decode_read_trace(mtp_decode_plan *P, uint64_t *out, int capacity, int *n_out) {
  MTP_REQUIRE(P && out && n_out && capacity >= P->n_trace, "bad arguments (capacity below the trace size)");
  if (cudaMemcpy(out, P->trace_buf, sizeof(uint64_t) * P->n_trace, cudaMemcpyDeviceToHost) != cudaSuccess)
    return fail(MTP_ERR_CUDA, "reading the decode trace failed");
  *n_out = P->n_trace;
  return MTP_OK;
}

void mtp_decode_cache_destroy(mtp_decode_cache *c) {
  if (!c) return;
  cudaFree(c->d_cache);
  delete c;
}

void mtp_decode_plan_destroy(mtp_decode_plan *P) {
  if (!P) return;
  cudaFree(P->scratch);
  delete P;
}

}  // extern "C"
