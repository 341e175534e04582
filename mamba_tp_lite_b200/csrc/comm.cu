// Row-parallel reductions over NVLink peer memory, with the reference's wire formats.
//
// Modes (mamba_lite/tp_utils.py):
//   fp32     all_reduce_sum            :23-28   ranks' fp32 partials summed in rank order
//   fp16     all_reduce_sum_fp16       :31-42   fp16 on the wire, fp32 rank-ordered sum, one fp16 rounding
//   int8tok  all_reduce_sum_int8_gather_tok :103-131, :145-149
//            per row: scale = max(amax, 1e-8)/127, q = clamp(rint(x/scale), +-127);
//            slot payload [rows*4 scale bytes | rows*cols int8] exactly as tp_utils.py:113;
//            result = sum_r float(q_r) * s_r from zeros, in rank order (product rounded, then add).
//
// Transport: every rank's comm allocation is mapped by its peers through CUDA IPC.  A reduction
// kernel of G CTAs runs on every rank; CTA j owns the same rows on every rank.
//   one-shot (small):  push wire rows to every rank's slot[my_rank] -> flag -> wait for all ranks'
//                      CTA j -> every rank reduces all its rows itself (identical order => identical bits)
//   two-shot (large):  push each wire row only to the row's owner rank (rows split in ws chunks) ->
//                      flag -> owner reduces its rows and pushes the fp32 result row to every rank's
//                      gather buffer -> flag -> every rank runs the epilogue on the gathered rows.
// Flag values come from a per-site epoch counter in device memory: every CTA of a call reads it at
// start and the last CTA to finish advances it, so a captured CUDA graph replays correctly and all
// ranks agree on it.  Receive slots are double-buffered by epoch parity: a rank can run at most one
// call ahead of a peer, so consecutive calls on one site never write a slot a peer still reads.  Each wait is bounded (globaltimer); on expiry
// the kernel stores MTP_ERR_TIMEOUT in the context's status word and returns.
#include <cstdlib>
#include <cstring>
#include <vector>
#include "common.cuh"
#include "comm_dev.cuh"
#include "wire.cuh"

namespace mtp {

constexpr int WPB = 8;  // warps (rows in flight) per CTA

// ----------------------------------------------------------------- device helpers
__device__ __forceinline__ float warp_max(float v) {
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}


// Row amax of a fp32 row (warp).
__device__ __forceinline__ float row_amax(const float *row, int cols, int lane) {
  float m = 0.f;
  for (int c = lane; c < cols; c += 32) m = fmaxf(m, fabsf(row[c]));
  return warp_max(m);
}

// Write one row's wire representation to slot `dst` (a rank's receive slot base for this call).
template <int MODE>
__device__ __forceinline__ void write_wire_row(char *dst, const float *row, int r, int rows, int cols, int lane,
                                               float scale) {
  if (MODE == MTP_RED_FP32) {
    float *o = reinterpret_cast<float *>(dst) + (size_t)r * cols;
    if ((cols & 3) == 0) {
      for (int c = lane * 4; c < cols; c += 128) *reinterpret_cast<float4 *>(o + c) = *reinterpret_cast<const float4 *>(row + c);
    } else {
      for (int c = lane; c < cols; c += 32) o[c] = row[c];
    }
  } else if (MODE == MTP_RED_FP16) {
    __half *o = reinterpret_cast<__half *>(dst) + (size_t)r * cols;
    if ((cols & 3) == 0) {
      for (int c = lane * 4; c < cols; c += 128) {
        const float4 v = *reinterpret_cast<const float4 *>(row + c);
        __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t *>(&a);
        u.y = *reinterpret_cast<uint32_t *>(&b);
        *reinterpret_cast<uint2 *>(o + c) = u;
      }
    } else {
      for (int c = lane; c < cols; c += 32) o[c] = __float2half_rn(row[c]);
    }
  } else {
    float *sc = reinterpret_cast<float *>(dst);
    int8_t *q = reinterpret_cast<int8_t *>(dst + (size_t)4 * rows) + (size_t)r * cols;
    if (lane == 0) sc[r] = scale;
    if ((cols & 3) == 0) {
      for (int c = lane * 4; c < cols; c += 128) {
        const float4 v = *reinterpret_cast<const float4 *>(row + c);
        *reinterpret_cast<uint32_t *>(q + c) = pack4(quant1(v.x, scale), quant1(v.y, scale), quant1(v.z, scale), quant1(v.w, scale));
      }
    } else {
      for (int c = lane; c < cols; c += 32) q[c] = (int8_t)quant1(row[c], scale);
    }
  }
}

// Rank-ordered reduction of row r over `nsrc` wire slots; writes the fp32 result row to `out`.
template <int MODE>
__device__ __forceinline__ void reduce_row(char *const *slots, int nsrc, int r, int rows, int cols, int lane, float *out) {
  if (MODE == MTP_RED_INT8TOK) {
    float s[MAX_WS];
    for (int k = 0; k < nsrc; ++k) s[k] = __ldcg(reinterpret_cast<const float *>(slots[k]) + r);
    if ((cols & 3) == 0) {
      for (int c = lane * 4; c < cols; c += 128) {
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
        for (int k = 0; k < nsrc; ++k) {
          const uint32_t w = __ldcg(reinterpret_cast<const unsigned int *>(slots[k] + (size_t)4 * rows + (size_t)r * cols + c));
          a0 = __fadd_rn(a0, __fmul_rn(unpack_i8(w, 0), s[k]));
          a1 = __fadd_rn(a1, __fmul_rn(unpack_i8(w, 1), s[k]));
          a2 = __fadd_rn(a2, __fmul_rn(unpack_i8(w, 2), s[k]));
          a3 = __fadd_rn(a3, __fmul_rn(unpack_i8(w, 3), s[k]));
        }
        *reinterpret_cast<float4 *>(out + c) = make_float4(a0, a1, a2, a3);
      }
    } else {
      for (int c = lane; c < cols; c += 32) {
        float a = 0.f;
        for (int k = 0; k < nsrc; ++k) {
          const int8_t q = *(const volatile int8_t *)(slots[k] + (size_t)4 * rows + (size_t)r * cols + c);
          a = __fadd_rn(a, __fmul_rn((float)q, s[k]));
        }
        out[c] = a;
      }
    }
  } else if (MODE == MTP_RED_FP16) {
    for (int c = lane; c < cols; c += 32) {
      float a = 0.f;
      for (int k = 0; k < nsrc; ++k) {
        const unsigned short u = __ldcg(reinterpret_cast<const unsigned short *>(slots[k]) + (size_t)r * cols + c);
        a = __fadd_rn(a, __half2float(__ushort_as_half(u)));
      }
      out[c] = __half2float(__float2half_rn(a));
    }
  } else {
    if ((cols & 3) == 0) {
      for (int c = lane * 4; c < cols; c += 128) {
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int k = 0; k < nsrc; ++k) {
          const float4 v = __ldcg(reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(slots[k]) + (size_t)r * cols + c));
          a.x = __fadd_rn(a.x, v.x); a.y = __fadd_rn(a.y, v.y); a.z = __fadd_rn(a.z, v.z); a.w = __fadd_rn(a.w, v.w);
        }
        *reinterpret_cast<float4 *>(out + c) = a;
      }
    } else {
      for (int c = lane; c < cols; c += 32) {
        float a = 0.f;
        for (int k = 0; k < nsrc; ++k) a = __fadd_rn(a, __ldcg(reinterpret_cast<const float *>(slots[k]) + (size_t)r * cols + c));
        out[c] = a;
      }
    }
  }
}

// ----------------------------------------------------------------- epilogues
enum { EPI_PLAIN = 0, EPI_XPROJ = 1, EPI_OUTPROJ = 2 };

struct EpiOut {
  float *out;           // PLAIN: [rows, cols]
  void *dt_low;         // XPROJ: [rows, R] in dt_dtype
  float *bc;            // XPROJ: [rows, 2N]
  int R, dt_dtype;
  const void *bias;     // OUTPROJ (model dtype) or NULL
  float *resid;         // OUTPROJ [rows, D] in/out
  const void *norm_w;   // OUTPROJ
  void *normed;         // OUTPROJ [rows, D] or NULL
  float eps;
  int out_dtype;        // OUTPROJ: dtype of bias / norm_w / normed
  int rdt;              // dtype the reduced values are rounded to (the collective's return dtype)
  int wide;             // rows take the 16-column granule layout (RMSNorm sum order of WideOps)
};


__device__ __forceinline__ float ld_any(const void *p, int dtype, size_t i) {
  return dtype == MTP_F32 ? ((const float *)p)[i] : __bfloat162float(((const __nv_bfloat16 *)p)[i]);
}
__device__ __forceinline__ void st_any(void *p, int dtype, size_t i, float v) {
  if (dtype == MTP_F32) ((float *)p)[i] = v;
  else ((__nv_bfloat16 *)p)[i] = __float2bfloat16_rn(v);
}

// Sum of squares of 4 consecutive residual values, rounded explicitly so that every
// kernel variant that gives a lane the same columns computes the same RMS bits.
__device__ __forceinline__ float sq4(float4 h) {
  float t = __fmul_rn(h.x, h.x);
  t = __fmaf_rn(h.y, h.y, t);
  t = __fmaf_rn(h.z, h.z, t);
  return __fmaf_rn(h.w, h.w, t);
}

// `val` is the reduced row (fp32, in global scratch or the gather buffer); read with __ldcg.
// With cols % 4 == 0 lane l owns columns 4l + 128i .. +3, as the register-row kernel.
template <int EPI>
__device__ __forceinline__ void epilogue_row(const EpiOut &e, const float *val, int r, int cols, int lane) {
  if (EPI == EPI_OUTPROJ && e.wide) {
    // lane l owns the 16-column granules 16 (32 i + l), summed four values at a time in column
    // order: the order of the wide-row pipelined kernel, so both variants give the same bits
    float ss = 0.f;
    float *res = e.resid + (size_t)r * cols;
    for (int c0 = 16 * lane; c0 < cols; c0 += 512) {
      for (int q = 0; q < 16; q += 4) {
        const int c = c0 + q;
        float4 v = __ldcg(reinterpret_cast<const float4 *>(val + c));
        if (e.bias) {
          v.x += ld_any(e.bias, e.out_dtype, c); v.y += ld_any(e.bias, e.out_dtype, c + 1);
          v.z += ld_any(e.bias, e.out_dtype, c + 2); v.w += ld_any(e.bias, e.out_dtype, c + 3);
        }
        const float4 h0 = *reinterpret_cast<const float4 *>(res + c);
        const float4 h = make_float4(h0.x + v.x, h0.y + v.y, h0.z + v.z, h0.w + v.w);
        *reinterpret_cast<float4 *>(res + c) = h;
        ss = __fadd_rn(ss, sq4(h));
      }
    }
    if (e.normed) {
      const float rs = rsqrtf(warp_sum(ss) / (float)cols + e.eps);
      for (int c0 = 16 * lane; c0 < cols; c0 += 512) {
        for (int q = 0; q < 16; ++q) {
          const int c = c0 + q;
          st_any(e.normed, e.out_dtype, (size_t)r * cols + c, ld_any(e.norm_w, e.out_dtype, c) * (res[c] * rs));
        }
      }
    }
    return;
  }
  if (EPI == EPI_OUTPROJ && (cols & 3) == 0) {
    float ss = 0.f;
    float *res = e.resid + (size_t)r * cols;
    for (int c = lane * 4; c < cols; c += 128) {
      float4 v = __ldcg(reinterpret_cast<const float4 *>(val + c));
      if (e.bias) {
        v.x += ld_any(e.bias, e.out_dtype, c); v.y += ld_any(e.bias, e.out_dtype, c + 1);
        v.z += ld_any(e.bias, e.out_dtype, c + 2); v.w += ld_any(e.bias, e.out_dtype, c + 3);
      }
      const float4 h0 = *reinterpret_cast<const float4 *>(res + c);
      const float4 h = make_float4(h0.x + v.x, h0.y + v.y, h0.z + v.z, h0.w + v.w);
      *reinterpret_cast<float4 *>(res + c) = h;
      ss = __fadd_rn(ss, sq4(h));
    }
    if (e.normed) {
      const float rs = rsqrtf(warp_sum(ss) / (float)cols + e.eps);
      for (int c = lane * 4; c < cols; c += 128) {
        const float4 h = *reinterpret_cast<const float4 *>(res + c);
        const float hv[4] = {h.x, h.y, h.z, h.w};
#pragma unroll
        for (int q = 0; q < 4; ++q)
          st_any(e.normed, e.out_dtype, (size_t)r * cols + c + q, ld_any(e.norm_w, e.out_dtype, c + q) * (hv[q] * rs));
      }
    }
    return;
  }
  if (EPI == EPI_PLAIN) {
    for (int c = lane; c < cols; c += 32) e.out[(size_t)r * cols + c] = __ldcg(val + c);
  } else if (EPI == EPI_XPROJ) {
    for (int c = lane; c < cols; c += 32) {
      const float v = __ldcg(val + c);
      if (c < e.R) st_any(e.dt_low, e.dt_dtype, (size_t)r * e.R + c, v);
      else e.bc[(size_t)r * (cols - e.R) + (c - e.R)] = v;
    }
  } else {
    float ss = 0.f;
    float *res = e.resid + (size_t)r * cols;
    for (int c = lane; c < cols; c += 32) {
      float v = __ldcg(val + c);
      if (e.bias) v = v + ld_any(e.bias, e.out_dtype, c);
      const float h = res[c] + v;
      res[c] = h;
      ss += h * h;
    }
    if (e.normed) {
      ss = warp_sum(ss);
      const float rs = rsqrtf(ss / (float)cols + e.eps);
      for (int c = lane; c < cols; c += 32)
        st_any(e.normed, e.out_dtype, (size_t)r * cols + c, ld_any(e.norm_w, e.out_dtype, c) * (res[c] * rs));
    }
  }
}

// ----------------------------------------------------------------- flags

// Signal phase `phase` of CTA j to `targets` (bitmask of ranks), after all threads' stores:
// the CTA barrier orders every thread's stores before the flag-writing threads, whose
// system-scope fence and release store then publish them (one fence per target rank, not
// one per thread: a system fence waits for the thread's outstanding remote stores).
__device__ __forceinline__ void signal(const CommDev &d, int site, int phase, uint32_t epoch, uint32_t targets) {
  __syncthreads();
  if (threadIdx.x < (unsigned)d.ws && (targets >> threadIdx.x) & 1u) {
    __threadfence_system();
    st_release_sys(flag_ptr(d.peer[threadIdx.x], d, site, phase, d.rank, blockIdx.x), epoch);
  }
}

// Wait until every rank in `sources` signalled phase `phase` of CTA j.  Returns false on timeout.
__device__ __forceinline__ bool wait_all(const CommDev &d, int site, int phase, uint32_t epoch, uint32_t sources,
                                         int *abort_sm) {
  if (threadIdx.x < (unsigned)d.ws && (sources >> threadIdx.x) & 1u) {
    const uint32_t *f = flag_ptr(d.peer[d.rank], d, site, phase, threadIdx.x, blockIdx.x);
    const unsigned long long t0 = globaltimer_ns();
    uint32_t it = 0;
    while ((int)(ld_acquire_sys(f) - epoch) < 0) {
      if ((++it & 63u) == 0 && globaltimer_ns() - t0 > d.timeout_ns) {
        atomicExch(reinterpret_cast<int *>(d.peer[d.rank] + d.off_status), MTP_ERR_TIMEOUT);
        *abort_sm = 1;
        break;
      }
    }
    __threadfence();
  }
  // the acquiring threads' loads, then the barrier, order the peers' data before every
  // thread's reads
  __syncthreads();
  return *abort_sm == 0;
}

// ----------------------------------------------------------------- the reduction kernel
// partial: [rows, cols] fp32 local.  scratch: [G*WPB, cols] fp32 per-warp row scratch (world size 1 and one-shot).
template <int MODE, int EPI>
__global__ void __launch_bounds__(WPB * 32) reduce_kernel(CommDev d, bool has_comm, int site, const float *__restrict__ partial,
                                                          int rows, int cols, bool two_shot, float *scratch, EpiOut e) {
  MTP_PDL_WAIT();
  MTP_PDL_TRIGGER();
  __shared__ int abort_sm;
  __shared__ uint32_t epoch_sm;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = blockIdx.x, G = gridDim.x;
  float *wrow = scratch + (size_t)(j * WPB + warp) * cols;
  if (!has_comm) {
    // world size 1: the wire round trip alone (fp16 cast / int8 quantise-dequantise)
    for (int r = j * WPB + warp; r < rows; r += G * WPB) {
      const float *row = partial + (size_t)r * cols;
      if (MODE == MTP_RED_FP32) {
        for (int c = lane; c < cols; c += 32) wrow[c] = rnd_rdt(row[c], e.rdt);
      } else if (MODE == MTP_RED_FP16) {
        for (int c = lane; c < cols; c += 32) wrow[c] = rnd_rdt(__half2float(__float2half_rn(row[c])), e.rdt);
      } else {
        const float sc = row_scale(row_amax(row, cols, lane));
        for (int c = lane; c < cols; c += 32)
          wrow[c] = rnd_rdt(__fadd_rn(0.f, __fmul_rn((float)quant1(row[c], sc), sc)), e.rdt);
      }
      __syncwarp();
      epilogue_row<EPI>(e, wrow, r, cols, lane);
      __syncwarp();
    }
    return;
  }
  uint32_t *ep = reinterpret_cast<uint32_t *>(d.peer[d.rank] + d.off_epoch) + site;
  if (threadIdx.x == 0) {
    abort_sm = 0;
    epoch_sm = *reinterpret_cast<volatile uint32_t *>(ep) + 1u;
  }
  __syncthreads();
  const uint32_t epoch = epoch_sm;
  // the last CTA to leave publishes the epoch for the next call
  auto finish = [&]() {
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      unsigned int *done = reinterpret_cast<unsigned int *>(d.peer[d.rank] + d.off_done) + site;
      if (atomicAdd(done, 1u) == (unsigned)G - 1u) {
        *done = 0u;
        *reinterpret_cast<volatile uint32_t *>(ep) = epoch;
        __threadfence();
      }
    }
  };
  const size_t half = (size_t)(epoch & 1u) * d.ws * d.slot_bytes[site];
  const uint32_t all = (1u << d.ws) - 1u;
  const int chunk = (rows + d.ws - 1) / d.ws;  // two-shot ownership: rows [k*chunk, (k+1)*chunk) -> rank k
  // phase 0: push wire rows
  for (int r = j * WPB + warp; r < rows; r += G * WPB) {
    const float *row = partial + (size_t)r * cols;
    const float sc = MODE == MTP_RED_INT8TOK ? row_scale(row_amax(row, cols, lane)) : 0.f;
    if (two_shot) {
      const int owner = r / chunk;
      write_wire_row<MODE>(d.peer[owner] + d.off_recv[site] + half + (size_t)d.rank * d.slot_bytes[site], row, r, rows, cols, lane, sc);
    } else {
      for (int k = 0; k < d.ws; ++k) {
        const int dst = (d.rank + k) % d.ws;  // stagger destinations across ranks
        write_wire_row<MODE>(d.peer[dst] + d.off_recv[site] + half + (size_t)d.rank * d.slot_bytes[site], row, r, rows, cols, lane, sc);
      }
    }
  }
  signal(d, site, 0, epoch, all);
  if (!wait_all(d, site, 0, epoch, all, &abort_sm)) { finish(); return; }
  char *slots[MAX_WS];
  for (int k = 0; k < d.ws; ++k) slots[k] = d.peer[d.rank] + d.off_recv[site] + half + (size_t)k * d.slot_bytes[site];
  if (!two_shot) {
    for (int r = j * WPB + warp; r < rows; r += G * WPB) {
      reduce_row<MODE>(slots, d.ws, r, rows, cols, lane, wrow);
      __syncwarp();
      for (int c = lane; c < cols; c += 32) wrow[c] = rnd_rdt(wrow[c], e.rdt);
      __syncwarp();
      epilogue_row<EPI>(e, wrow, r, cols, lane);
      __syncwarp();
    }
    finish();
    return;
  }
  // phase 1 (owner): reduce owned rows, push fp32 result rows to every rank's gather buffer
  float *gath_local = reinterpret_cast<float *>(d.peer[d.rank] + d.off_gath[site]);
  for (int r = j * WPB + warp; r < rows; r += G * WPB) {
    if (r / chunk != d.rank) continue;
    float *mine = gath_local + (size_t)r * cols;
    reduce_row<MODE>(slots, d.ws, r, rows, cols, lane, mine);
    __syncwarp();
    for (int c = lane; c < cols; c += 32) mine[c] = rnd_rdt(mine[c], e.rdt);
    __syncwarp();
    for (int k = 1; k < d.ws; ++k) {
      const int dst = (d.rank + k) % d.ws;
      float *o = reinterpret_cast<float *>(d.peer[dst] + d.off_gath[site]) + (size_t)r * cols;
      if ((cols & 3) == 0) {
        for (int c = lane * 4; c < cols; c += 128) *reinterpret_cast<float4 *>(o + c) = *reinterpret_cast<const float4 *>(mine + c);
      } else {
        for (int c = lane; c < cols; c += 32) o[c] = mine[c];
      }
    }
  }
  signal(d, site, 1, epoch, all);
  if (!wait_all(d, site, 1, epoch, all, &abort_sm)) { finish(); return; }
  for (int r = j * WPB + warp; r < rows; r += G * WPB) epilogue_row<EPI>(e, gath_local + (size_t)r * cols, r, cols, lane);
  finish();
}

// ----------------------------------------------------------------- register-row reduction
// One warp per row; the row lives in registers as VPL float4 chunks per lane
// (columns 4*(i*32+lane) .. +3 of chunk i), so the quantiser, the wire writes,
// the rank-ordered reduce and the epilogue each touch memory once, with 16-byte
// (fp32), 8-byte (fp16) or 4-byte (int8) vector accesses.  Needs cols % 4 == 0
// and cols <= 128 * VPL.
template <int VPL> struct RowV { float4 v[VPL]; };

template <bool CG, int VPL>
__device__ __forceinline__ void load_rowv(const float *row, int cols, int lane, RowV<VPL> &R) {
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (i * 32 + lane) * 4;
    if (c < cols) R.v[i] = CG ? __ldcg(reinterpret_cast<const float4 *>(row + c)) : *reinterpret_cast<const float4 *>(row + c);
    else R.v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

template <int VPL>
__device__ __forceinline__ float rowv_amax(const RowV<VPL> &R) {
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) m = fmaxf(fmaxf(fmaxf(m, fabsf(R.v[i].x)), fmaxf(fabsf(R.v[i].y), fabsf(R.v[i].z))), fabsf(R.v[i].w));
  return warp_max(m);
}


// world size 1: the wire format's round trip alone, in registers
template <int MODE, int VPL>
__device__ __forceinline__ void roundtrip_v(RowV<VPL> &R) {
  if (MODE == MTP_RED_FP16) {
#pragma unroll
    for (int i = 0; i < VPL; ++i) R.v[i] = make_float4(h1(R.v[i].x), h1(R.v[i].y), h1(R.v[i].z), h1(R.v[i].w));
  } else if (MODE == MTP_RED_INT8TOK) {
    const float s = row_scale(rowv_amax(R));
#pragma unroll
    for (int i = 0; i < VPL; ++i) R.v[i] = make_float4(dq1(R.v[i].x, s), dq1(R.v[i].y, s), dq1(R.v[i].z, s), dq1(R.v[i].w, s));
  }
}

template <int MODE, int VPL>
__device__ __forceinline__ void write_wire_v(char *dst, const RowV<VPL> &R, int r, int rows, int cols, int lane, float scale) {
  if (MODE == MTP_RED_INT8TOK && lane == 0) reinterpret_cast<float *>(dst)[r] = scale;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (i * 32 + lane) * 4;
    if (c >= cols) break;
    const float4 v = R.v[i];
    if (MODE == MTP_RED_FP32) {
      *reinterpret_cast<float4 *>(reinterpret_cast<float *>(dst) + (size_t)r * cols + c) = v;
    } else if (MODE == MTP_RED_FP16) {
      __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
      uint2 u;
      u.x = *reinterpret_cast<uint32_t *>(&a);
      u.y = *reinterpret_cast<uint32_t *>(&b);
      *reinterpret_cast<uint2 *>(reinterpret_cast<__half *>(dst) + (size_t)r * cols + c) = u;
    } else {
      *reinterpret_cast<uint32_t *>(dst + (size_t)4 * rows + (size_t)r * cols + c) =
          pack4(quant1(v.x, scale), quant1(v.y, scale), quant1(v.z, scale), quant1(v.w, scale));
    }
  }
}

// rank-ordered reduction of row r over the slots, into registers
template <int MODE, int VPL>
__device__ __forceinline__ void reduce_v(char *const *slots, int nsrc, int r, int rows, int cols, int lane, RowV<VPL> &R) {
  float s[MAX_WS];
  if (MODE == MTP_RED_INT8TOK)
    for (int k = 0; k < nsrc; ++k) s[k] = __ldcg(reinterpret_cast<const float *>(slots[k]) + r);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (i * 32 + lane) * 4;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c < cols) {
      for (int k = 0; k < nsrc; ++k) {
        float4 v;
        if (MODE == MTP_RED_FP32) {
          v = __ldcg(reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(slots[k]) + (size_t)r * cols + c));
        } else if (MODE == MTP_RED_FP16) {
          const uint2 u = __ldcg(reinterpret_cast<const uint2 *>(reinterpret_cast<const __half *>(slots[k]) + (size_t)r * cols + c));
          const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
          const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
          v = make_float4(lo.x, lo.y, hi.x, hi.y);
        } else {
          const uint32_t w = __ldcg(reinterpret_cast<const unsigned int *>(slots[k] + (size_t)4 * rows + (size_t)r * cols + c));
          v = make_float4(__fmul_rn(unpack_i8(w, 0), s[k]), __fmul_rn(unpack_i8(w, 1), s[k]),
                          __fmul_rn(unpack_i8(w, 2), s[k]), __fmul_rn(unpack_i8(w, 3), s[k]));
        }
        a.x = __fadd_rn(a.x, v.x); a.y = __fadd_rn(a.y, v.y); a.z = __fadd_rn(a.z, v.z); a.w = __fadd_rn(a.w, v.w);
      }
      if (MODE == MTP_RED_FP16) a = make_float4(h1(a.x), h1(a.y), h1(a.z), h1(a.w));
    }
    R.v[i] = a;
  }
}

template <int VPL>
__device__ __forceinline__ void round_v(RowV<VPL> &R, int rdt) {
  if (rdt != MTP_BF16) return;
#pragma unroll
  for (int i = 0; i < VPL; ++i)
    R.v[i] = make_float4(rnd_rdt(R.v[i].x, rdt), rnd_rdt(R.v[i].y, rdt), rnd_rdt(R.v[i].z, rdt), rnd_rdt(R.v[i].w, rdt));
}

// gather rows travel in the result dtype: bf16 (8 bytes per 4 values) or fp32
template <int VPL>
__device__ __forceinline__ void store_gather_v(char *g, const RowV<VPL> &R, int r, int cols, int lane, int rdt) {
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (i * 32 + lane) * 4;
    if (c >= cols) break;
    if (rdt == MTP_BF16) {
      __nv_bfloat162 a = __floats2bfloat162_rn(R.v[i].x, R.v[i].y), b = __floats2bfloat162_rn(R.v[i].z, R.v[i].w);
      uint2 u;
      u.x = *reinterpret_cast<uint32_t *>(&a);
      u.y = *reinterpret_cast<uint32_t *>(&b);
      *reinterpret_cast<uint2 *>(reinterpret_cast<__nv_bfloat16 *>(g) + (size_t)r * cols + c) = u;
    } else {
      *reinterpret_cast<float4 *>(reinterpret_cast<float *>(g) + (size_t)r * cols + c) = R.v[i];
    }
  }
}
template <int VPL>
__device__ __forceinline__ void load_gather_v(const char *g, RowV<VPL> &R, int r, int cols, int lane, int rdt) {
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (i * 32 + lane) * 4;
    if (c >= cols) { R.v[i] = make_float4(0.f, 0.f, 0.f, 0.f); continue; }
    if (rdt == MTP_BF16) {
      const uint2 u = __ldcg(reinterpret_cast<const uint2 *>(reinterpret_cast<const __nv_bfloat16 *>(g) + (size_t)r * cols + c));
      const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.x));
      const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.y));
      R.v[i] = make_float4(lo.x, lo.y, hi.x, hi.y);
    } else {
      R.v[i] = __ldcg(reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(g) + (size_t)r * cols + c));
    }
  }
}

// The out_proj epilogue on a register row (narrow layout): bias, residual add (resid
// updated in place), then, when normed is requested, R = norm_w * (h * rsqrt(mean(h^2)
// + eps)) in fp32 (else R = h).  store_rows_v stores R in the output dtype.
template <int VPL>
__device__ __forceinline__ void outproj_norm_v(const EpiOut &e, RowV<VPL> &R, int r, int cols, int lane) {
  float ss = 0.f;
  float *res = e.resid + (size_t)r * cols;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (i * 32 + lane) * 4;
    if (c >= cols) break;
    float4 v = R.v[i];
    if (e.bias) {
      v.x += ld_any(e.bias, e.out_dtype, c); v.y += ld_any(e.bias, e.out_dtype, c + 1);
      v.z += ld_any(e.bias, e.out_dtype, c + 2); v.w += ld_any(e.bias, e.out_dtype, c + 3);
    }
    const float4 h0 = *reinterpret_cast<const float4 *>(res + c);
    const float4 h = make_float4(h0.x + v.x, h0.y + v.y, h0.z + v.z, h0.w + v.w);
    *reinterpret_cast<float4 *>(res + c) = h;
    ss = __fadd_rn(ss, sq4(h));
    R.v[i] = h;
  }
  if (!e.normed) return;
  const float rs = rsqrtf(warp_sum(ss) / (float)cols + e.eps);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (i * 32 + lane) * 4;
    if (c >= cols) break;
    const float4 h = R.v[i];
    float o[4] = {h.x * rs, h.y * rs, h.z * rs, h.w * rs};
#pragma unroll
    for (int q = 0; q < 4; ++q) o[q] = ld_any(e.norm_w, e.out_dtype, c + q) * o[q];
    R.v[i] = make_float4(o[0], o[1], o[2], o[3]);
  }
}

template <int VPL>
__device__ __forceinline__ void store_rows_v(void *dst, int dtype, const RowV<VPL> &R, int r, int cols, int lane) {
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (i * 32 + lane) * 4;
    if (c >= cols) break;
    const float4 o = R.v[i];
    if (dtype == MTP_F32) {
      *reinterpret_cast<float4 *>(reinterpret_cast<float *>(dst) + (size_t)r * cols + c) = o;
    } else {
      __nv_bfloat162 a = __floats2bfloat162_rn(o.x, o.y), b = __floats2bfloat162_rn(o.z, o.w);
      uint2 u;
      u.x = *reinterpret_cast<uint32_t *>(&a);
      u.y = *reinterpret_cast<uint32_t *>(&b);
      *reinterpret_cast<uint2 *>(reinterpret_cast<__nv_bfloat16 *>(dst) + (size_t)r * cols + c) = u;
    }
  }
}

template <int EPI, int VPL>
__device__ __forceinline__ void epilogue_v(const EpiOut &e, RowV<VPL> &R, int r, int cols, int lane) {
  if (EPI == EPI_PLAIN) {
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c = (i * 32 + lane) * 4;
      if (c < cols) *reinterpret_cast<float4 *>(e.out + (size_t)r * cols + c) = R.v[i];
    }
  } else if (EPI == EPI_XPROJ) {
    const int n2 = cols - e.R;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c = (i * 32 + lane) * 4;
      if (c >= cols) break;
      const float v[4] = {R.v[i].x, R.v[i].y, R.v[i].z, R.v[i].w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int cc = c + q;
        if (cc < e.R) st_any(e.dt_low, e.dt_dtype, (size_t)r * e.R + cc, v[q]);
        else e.bc[(size_t)r * n2 + (cc - e.R)] = v[q];
      }
    }
  } else {
    outproj_norm_v(e, R, r, cols, lane);
    if (e.normed) store_rows_v(e.normed, e.out_dtype, R, r, cols, lane);
  }
}

// ----------------------------------------------------------------- wide-row reduction (16-column granules)
// For rows of at least 512 values with cols % 16 == 0 (the out_proj site: d_model 768 ..
// 2560): lane l of a warp owns the 16 consecutive columns 16 (32 i + l) .. +15 of chunk
// i, so every global access is 16 bytes or more per lane: the fp32 partial and the
// residual as four float4, the int8 wire as one 16-byte word, the fp16 wire and the bf16
// gather / normed rows as two.  The int8 slot keeps the reference's payload order
// (scales, then rows x cols int8) with the int8 block starting at the next 16-byte
// boundary.  NC chunks per lane: cols <= 512 NC.
template <int NC> struct RowW { float v[NC][16]; };

__device__ __forceinline__ size_t q_offset(int rows) { return ((size_t)4 * rows + 15) & ~(size_t)15; }

template <bool CG, int NC>
__device__ __forceinline__ void load_roww(const float *row, int cols, int lane, RowW<NC> &R) {
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = 16 * (i * 32 + lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
      if (c < cols) f = CG ? __ldcg(reinterpret_cast<const float4 *>(row + c) + j) : *(reinterpret_cast<const float4 *>(row + c) + j);
      R.v[i][4 * j] = f.x; R.v[i][4 * j + 1] = f.y; R.v[i][4 * j + 2] = f.z; R.v[i][4 * j + 3] = f.w;
    }
  }
}

template <int NC>
__device__ __forceinline__ float roww_amax(const RowW<NC> &R) {
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < NC; ++i)
#pragma unroll
    for (int k = 0; k < 16; ++k) m = fmaxf(m, fabsf(R.v[i][k]));
  return warp_max(m);
}

template <int MODE, int NC>
__device__ __forceinline__ void roundtrip_w(RowW<NC> &R) {
  if (MODE == MTP_RED_FP16) {
#pragma unroll
    for (int i = 0; i < NC; ++i)
#pragma unroll
      for (int k = 0; k < 16; ++k) R.v[i][k] = h1(R.v[i][k]);
  } else if (MODE == MTP_RED_INT8TOK) {
    const float s = row_scale(roww_amax(R));
#pragma unroll
    for (int i = 0; i < NC; ++i)
#pragma unroll
      for (int k = 0; k < 16; ++k) R.v[i][k] = dq1(R.v[i][k], s);
  }
}

template <int NC>
__device__ __forceinline__ void round_w(RowW<NC> &R, int rdt) {
  if (rdt != MTP_BF16) return;
#pragma unroll
  for (int i = 0; i < NC; ++i)
#pragma unroll
    for (int k = 0; k < 16; ++k) R.v[i][k] = rnd_rdt(R.v[i][k], rdt);
}

__device__ __forceinline__ uint4 pack_bf16x8(const float *v) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t *>(&h2);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
__device__ __forceinline__ void unpack_bf16x8(uint4 u, float *v) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[i]));
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ uint4 pack_half8(const float *v) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h2 = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t *>(&h2);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
__device__ __forceinline__ void unpack_half8(uint4 u, float *v) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

template <int MODE, int NC>
__device__ __forceinline__ void write_wire_w(char *dst, const RowW<NC> &R, int r, int rows, int cols, int lane,
                                             float scale) {
  if (MODE == MTP_RED_INT8TOK && lane == 0) reinterpret_cast<float *>(dst)[r] = scale;
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = 16 * (i * 32 + lane);
    if (c >= cols) break;
    const float *v = R.v[i];
    if (MODE == MTP_RED_FP32) {
      float4 *o = reinterpret_cast<float4 *>(reinterpret_cast<float *>(dst) + (size_t)r * cols + c);
#pragma unroll
      for (int j = 0; j < 4; ++j) o[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    } else if (MODE == MTP_RED_FP16) {
      uint4 *o = reinterpret_cast<uint4 *>(reinterpret_cast<__half *>(dst) + (size_t)r * cols + c);
      o[0] = pack_half8(v);
      o[1] = pack_half8(v + 8);
    } else {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        w[j] = pack4(quant1(v[4 * j], scale), quant1(v[4 * j + 1], scale), quant1(v[4 * j + 2], scale),
                     quant1(v[4 * j + 3], scale));
      *reinterpret_cast<uint4 *>(dst + q_offset(rows) + (size_t)r * cols + c) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// Rank-ordered reduction of row r over the slots into registers (16-byte loads per source
// and granule; sums in rank order, product rounded before the add for int8).
template <int MODE, int NC>
__device__ __forceinline__ void reduce_w(char *const *slots, int nsrc, int r, int rows, int cols, int lane,
                                         RowW<NC> &R) {
#pragma unroll
  for (int i = 0; i < NC; ++i)
#pragma unroll
    for (int k = 0; k < 16; ++k) R.v[i][k] = 0.f;
  for (int k = 0; k < nsrc; ++k) {
    const float sk = MODE == MTP_RED_INT8TOK ? __ldcg(reinterpret_cast<const float *>(slots[k]) + r) : 0.f;
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const int c = 16 * (i * 32 + lane);
      if (c >= cols) break;
      float *a = R.v[i];
      if (MODE == MTP_RED_INT8TOK) {
        const uint4 w = __ldcg(reinterpret_cast<const uint4 *>(slots[k] + q_offset(rows) + (size_t)r * cols + c));
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 16; ++j) a[j] = __fadd_rn(a[j], __fmul_rn(unpack_i8(ww[j >> 2], j & 3), sk));
      } else if (MODE == MTP_RED_FP16) {
        const uint4 *p = reinterpret_cast<const uint4 *>(reinterpret_cast<const __half *>(slots[k]) + (size_t)r * cols + c);
        float f[16];
        unpack_half8(__ldcg(p), f);
        unpack_half8(__ldcg(p + 1), f + 8);
#pragma unroll
        for (int j = 0; j < 16; ++j) a[j] = __fadd_rn(a[j], f[j]);
      } else {
        const float4 *p = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(slots[k]) + (size_t)r * cols + c);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float4 f = __ldcg(p + j);
          a[4 * j] = __fadd_rn(a[4 * j], f.x); a[4 * j + 1] = __fadd_rn(a[4 * j + 1], f.y);
          a[4 * j + 2] = __fadd_rn(a[4 * j + 2], f.z); a[4 * j + 3] = __fadd_rn(a[4 * j + 3], f.w);
        }
      }
    }
  }
  if (MODE == MTP_RED_FP16) {
#pragma unroll
    for (int i = 0; i < NC; ++i)
#pragma unroll
      for (int k = 0; k < 16; ++k) R.v[i][k] = h1(R.v[i][k]);
  }
}

// gather rows travel in the result dtype (bf16: 32 bytes per granule, fp32: 64)
template <int NC>
__device__ __forceinline__ void store_gather_w(char *g, const RowW<NC> &R, int r, int cols, int lane, int rdt) {
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = 16 * (i * 32 + lane);
    if (c >= cols) break;
    if (rdt == MTP_BF16) {
      uint4 *o = reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(g) + (size_t)r * cols + c);
      o[0] = pack_bf16x8(R.v[i]);
      o[1] = pack_bf16x8(R.v[i] + 8);
    } else {
      float4 *o = reinterpret_cast<float4 *>(reinterpret_cast<float *>(g) + (size_t)r * cols + c);
#pragma unroll
      for (int j = 0; j < 4; ++j) o[j] = make_float4(R.v[i][4 * j], R.v[i][4 * j + 1], R.v[i][4 * j + 2], R.v[i][4 * j + 3]);
    }
  }
}
template <int NC>
__device__ __forceinline__ void load_gather_w(const char *g, RowW<NC> &R, int r, int cols, int lane, int rdt) {
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = 16 * (i * 32 + lane);
    if (c >= cols) {
#pragma unroll
      for (int k = 0; k < 16; ++k) R.v[i][k] = 0.f;
      continue;
    }
    if (rdt == MTP_BF16) {
      const uint4 *p = reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(g) + (size_t)r * cols + c);
      const uint4 a = __ldcg(p), b = __ldcg(p + 1);
      unpack_bf16x8(a, R.v[i]);
      unpack_bf16x8(b, R.v[i] + 8);
    } else {
      const float4 *p = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(g) + (size_t)r * cols + c);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 f = __ldcg(p + j);
        R.v[i][4 * j] = f.x; R.v[i][4 * j + 1] = f.y; R.v[i][4 * j + 2] = f.z; R.v[i][4 * j + 3] = f.w;
      }
    }
  }
}

// 16 consecutive values of a model-dtype (bf16) or fp32 vector starting at column c
__device__ __forceinline__ void load_vec16(const void *p, int dtype, int c, float *v) {
  if (dtype == MTP_F32) {
    const float4 *q = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(p) + c);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 f = __ldg(q + j);
      v[4 * j] = f.x; v[4 * j + 1] = f.y; v[4 * j + 2] = f.z; v[4 * j + 3] = f.w;
    }
  } else {
    const uint4 *q = reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(p) + c);
    unpack_bf16x8(__ldg(q), v);
    unpack_bf16x8(__ldg(q + 1), v + 8);
  }
}

// The out_proj epilogue in the 16-column layout (as outproj_norm_v): bias, residual add,
// then R = norm_w * (h * rs) when normed is requested; store_rows_w stores R.
template <int NC>
__device__ __forceinline__ void outproj_norm_w(const EpiOut &e, RowW<NC> &R, int r, int cols, int lane) {
  float ss = 0.f;
  float *res = e.resid + (size_t)r * cols;
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = 16 * (i * 32 + lane);
    if (c >= cols) break;
    if (e.bias) {
      float b[16];
      load_vec16(e.bias, e.out_dtype, c, b);
#pragma unroll
      for (int k = 0; k < 16; ++k) R.v[i][k] += b[k];
    }
    float4 *rp = reinterpret_cast<float4 *>(res + c);
    float4 h0[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) h0[j] = rp[j];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 h = make_float4(h0[j].x + R.v[i][4 * j], h0[j].y + R.v[i][4 * j + 1], h0[j].z + R.v[i][4 * j + 2],
                                   h0[j].w + R.v[i][4 * j + 3]);
      rp[j] = h;
      ss = __fadd_rn(ss, sq4(h));
      R.v[i][4 * j] = h.x; R.v[i][4 * j + 1] = h.y; R.v[i][4 * j + 2] = h.z; R.v[i][4 * j + 3] = h.w;
    }
  }
  if (!e.normed) return;
  const float rs = rsqrtf(warp_sum(ss) / (float)cols + e.eps);
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = 16 * (i * 32 + lane);
    if (c >= cols) break;
    float w[16];
    load_vec16(e.norm_w, e.out_dtype, c, w);
#pragma unroll
    for (int k = 0; k < 16; ++k) R.v[i][k] = w[k] * (R.v[i][k] * rs);
  }
}

template <int NC>
__device__ __forceinline__ void store_rows_w(void *dst, int dtype, const RowW<NC> &R, int r, int cols, int lane) {
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = 16 * (i * 32 + lane);
    if (c >= cols) break;
    if (dtype == MTP_F32) {
      float4 *p = reinterpret_cast<float4 *>(reinterpret_cast<float *>(dst) + (size_t)r * cols + c);
#pragma unroll
      for (int j = 0; j < 4; ++j) p[j] = make_float4(R.v[i][4 * j], R.v[i][4 * j + 1], R.v[i][4 * j + 2], R.v[i][4 * j + 3]);
    } else {
      uint4 *p = reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(dst) + (size_t)r * cols + c);
      p[0] = pack_bf16x8(R.v[i]);
      p[1] = pack_bf16x8(R.v[i] + 8);
    }
  }
}

// Epilogue of a reduced row in the 16-column layout.  The RMSNorm sum of squares runs over
// the lane's granules in column order, four values at a time (sq4), then across the warp:
// the same order as epilogue_row gives the wide layout, so every kernel variant computes the
// same bits.  Bias, norm_w and normed need 16-byte aligned rows (checked on the host).
template <int EPI, int NC>
__device__ __forceinline__ void epilogue_w(const EpiOut &e, RowW<NC> &R, int r, int cols, int lane) {
  if (EPI == EPI_PLAIN) {
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const int c = 16 * (i * 32 + lane);
      if (c >= cols) break;
      float4 *o = reinterpret_cast<float4 *>(e.out + (size_t)r * cols + c);
#pragma unroll
      for (int j = 0; j < 4; ++j) o[j] = make_float4(R.v[i][4 * j], R.v[i][4 * j + 1], R.v[i][4 * j + 2], R.v[i][4 * j + 3]);
    }
    return;
  }
  // EPI_OUTPROJ
  outproj_norm_w(e, R, r, cols, lane);
  if (e.normed) store_rows_w(e.normed, e.out_dtype, R, r, cols, lane);
}

// ----------------------------------------------------------------- pipelined reduction kernel
// Row operations of the two register layouts (narrow: float4 chunks, wide: 16-column
// granules), so one kernel body drives both.
template <int MODE_, int EPI_, int VPL>
struct NarrowOps {
  static constexpr int MODE = MODE_, EPI = EPI_, MINB = VPL >= 16 ? 2 : 3;
  using Row = RowV<VPL>;
  static __device__ __forceinline__ void load(const float *p, int cols, int lane, Row &R) { load_rowv<false>(p, cols, lane, R); }
  static __device__ __forceinline__ float amax(const Row &R) { return rowv_amax(R); }
  static __device__ __forceinline__ void roundtrip(Row &R) { roundtrip_v<MODE>(R); }
  static __device__ __forceinline__ void round(Row &R, int rdt) { round_v(R, rdt); }
  static __device__ __forceinline__ void wire(char *dst, const Row &R, int r, int rows, int cols, int lane, float sc) {
    write_wire_v<MODE>(dst, R, r, rows, cols, lane, sc);
  }
  static __device__ __forceinline__ void reduce(char *const *slots, int nsrc, int r, int rows, int cols, int lane, Row &R) {
    reduce_v<MODE>(slots, nsrc, r, rows, cols, lane, R);
  }
  static __device__ __forceinline__ void store_gather(char *g, const Row &R, int r, int cols, int lane, int rdt) {
    store_gather_v(g, R, r, cols, lane, rdt);
  }
  static __device__ __forceinline__ void load_gather(const char *g, Row &R, int r, int cols, int lane, int rdt) {
    load_gather_v(g, R, r, cols, lane, rdt);
  }
  static __device__ __forceinline__ void epilogue(const EpiOut &e, Row &R, int r, int cols, int lane) {
    epilogue_v<EPI>(e, R, r, cols, lane);
  }
  static __device__ __forceinline__ void norm(const EpiOut &e, Row &R, int r, int cols, int lane) {
    outproj_norm_v(e, R, r, cols, lane);
  }
  static __device__ __forceinline__ void store_normed(const EpiOut &e, const Row &R, int r, int cols, int lane) {
    store_rows_v(e.normed, e.out_dtype, R, r, cols, lane);
  }
};

template <int MODE_, int EPI_, int NC>
struct WideOps {
  static constexpr int MODE = MODE_, EPI = EPI_, MINB = 2;
  using Row = RowW<NC>;
  static __device__ __forceinline__ void load(const float *p, int cols, int lane, Row &R) { load_roww<false>(p, cols, lane, R); }
  static __device__ __forceinline__ float amax(const Row &R) { return roww_amax(R); }
  static __device__ __forceinline__ void roundtrip(Row &R) { roundtrip_w<MODE>(R); }
  static __device__ __forceinline__ void round(Row &R, int rdt) { round_w(R, rdt); }
  static __device__ __forceinline__ void wire(char *dst, const Row &R, int r, int rows, int cols, int lane, float sc) {
    write_wire_w<MODE>(dst, R, r, rows, cols, lane, sc);
  }
  static __device__ __forceinline__ void reduce(char *const *slots, int nsrc, int r, int rows, int cols, int lane, Row &R) {
    reduce_w<MODE>(slots, nsrc, r, rows, cols, lane, R);
  }
  static __device__ __forceinline__ void store_gather(char *g, const Row &R, int r, int cols, int lane, int rdt) {
    store_gather_w(g, R, r, cols, lane, rdt);
  }
  static __device__ __forceinline__ void load_gather(const char *g, Row &R, int r, int cols, int lane, int rdt) {
    load_gather_w(g, R, r, cols, lane, rdt);
  }
  static __device__ __forceinline__ void epilogue(const EpiOut &e, Row &R, int r, int cols, int lane) {
    epilogue_w<EPI>(e, R, r, cols, lane);
  }
  static __device__ __forceinline__ void norm(const EpiOut &e, Row &R, int r, int cols, int lane) {
    outproj_norm_w(e, R, r, cols, lane);
  }
  static __device__ __forceinline__ void store_normed(const EpiOut &e, const Row &R, int r, int cols, int lane) {
    store_rows_w(e.normed, e.out_dtype, R, r, cols, lane);
  }
};

// Flag phases of the pipelined protocol (phases 0 and 1 belong to the unpipelined
// scratch kernel and to the decode kernel, which flag with the bare epoch).
constexpr int PH_PUSH = 2, PH_GATHER = 3;
constexpr uint32_t ROUNDS_PER_EPOCH = 256;  // flag value of round k of a call: epoch * 256 + k

// Fence this thread's stores of the round, then flag `targets` for up to two (phase, value)
// pairs (the push round and the gather round of the two-shot pipeline).
__device__ __forceinline__ void signal_rounds(const CommDev &d, int site, int pa, uint32_t va, bool da, int pb,
                                              uint32_t vb, bool db) {
  __syncthreads();
  if (threadIdx.x < (unsigned)d.ws) {
    __threadfence_system();
    if (da) st_release_sys(flag_ptr(d.peer[threadIdx.x], d, site, pa, d.rank, blockIdx.x), va);
    if (db) st_release_sys(flag_ptr(d.peer[threadIdx.x], d, site, pb, d.rank, blockIdx.x), vb);
  }
}

// One reduction launch, pipelined in rounds.  CTA j owns the row slices s = 0, 1, ... with
// rows (s G + j) WPB + warp (the same rows on every rank); round k is slices
// [k rpw, (k+1) rpw).  One-shot: a round's wire rows go to every rank and are reduced one
// round later, after every rank's flag for that round -- so the NVLink transfer of round
// k overlaps the reduce and epilogue of round k-1.  Two-shot: round k's wire rows go to
// their owner rank (rows round-robin over the ranks); one round later the owner reduces
// them and pushes the rounded result rows to every rank's gather buffer; one round after
// that every rank runs the epilogue.  Every rank reduces in rank order, so all ranks hold
// the same bits.  Flag values grow with the round; every wait is bounded.
template <class Ops>
__global__ void __launch_bounds__(WPB * 32, Ops::MINB) reduce_pipe_kernel(CommDev d, bool has_comm, int site,
                                                                           const float *__restrict__ partial, int rows,
                                                                           int cols, bool two_shot, bool sp, int rpw,
                                                                           EpiOut e) {
  constexpr int MODE = Ops::MODE;
  MTP_PDL_WAIT();
  MTP_PDL_TRIGGER();
  __shared__ int abort_sm;
  __shared__ uint32_t epoch_sm;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = blockIdx.x, G = gridDim.x;
  typename Ops::Row R;
  const int S = rows > j * WPB ? (rows - j * WPB + G * WPB - 1) / (G * WPB) : 0;  // slices of this CTA
  auto row_of = [&](int sl) { return (sl * G + j) * WPB + warp; };
  if (!has_comm) {
    for (int sl = 0; sl < S; ++sl) {
      const int r = row_of(sl);
      if (r >= rows) continue;
      Ops::load(partial + (size_t)r * cols, cols, lane, R);
      Ops::roundtrip(R);
      Ops::round(R, e.rdt);
      Ops::epilogue(e, R, r, cols, lane);
    }
    return;
  }
  uint32_t *ep = reinterpret_cast<uint32_t *>(d.peer[d.rank] + d.off_epoch) + site;
  if (threadIdx.x == 0) {
    abort_sm = 0;
    epoch_sm = *reinterpret_cast<volatile uint32_t *>(ep) + 1u;
  }
  __syncthreads();
  const uint32_t epoch = epoch_sm;
  auto finish = [&]() {
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      unsigned int *done = reinterpret_cast<unsigned int *>(d.peer[d.rank] + d.off_done) + site;
      if (atomicAdd(done, 1u) == (unsigned)G - 1u) {
        *done = 0u;
        *reinterpret_cast<volatile uint32_t *>(ep) = epoch;
        __threadfence();
      }
    }
  };
  const size_t half = (size_t)(epoch & 1u) * d.ws * d.slot_bytes[site];
  const uint32_t all = (1u << d.ws) - 1u;
  // two-shot ownership: rows round-robin over the ranks, so in every round each CTA's
  // warps hold rows of every owner and each rank does 1/ws of the owner work of the round
  // (contiguous row chunks would give each round's rows to one or two ranks)
  auto owner_of = [&](int r) { return r % d.ws; };
  const size_t my_slot = d.off_recv[site] + half + (size_t)d.rank * d.slot_bytes[site];
  char *slots[MAX_WS];
  for (int k = 0; k < d.ws; ++k) slots[k] = d.peer[d.rank] + d.off_recv[site] + half + (size_t)k * d.slot_bytes[site];
  const int K = (S + rpw - 1) / rpw;
  const uint32_t v0 = epoch * ROUNDS_PER_EPOCH;
  // optional phase trace: thread 0 of CTA 0 and of the last CTA stamp each event
  unsigned long long *tr = nullptr;
  int tn = 0;
  if (d.trace && threadIdx.x == 0 && (j == 0 || j == G - 1)) {
    __shared__ unsigned int rec_sm;
    if (j == 0) rec_sm = atomicAdd(d.trace_count, 1u);
    else rec_sm = atomicAdd(d.trace_count + 1, 1u);
    unsigned long long *rec = d.trace + (size_t)(rec_sm % (unsigned)d.trace_cap) * TRACE_WORDS;
    if (j == 0) { rec[0] = G; rec[1] = K; rec[2] = (unsigned long long)two_shot | ((unsigned long long)site << 8); }
    tr = rec + 3 + (j == 0 ? 0 : 64);
    tr[tn++] = globaltimer_ns();
  }
  auto stamp = [&]() {
    if (tr && tn < 64) tr[tn++] = globaltimer_ns();
  };
  auto push_round = [&](int k) {
    for (int i = 0; i < rpw; ++i) {
      const int sl = k * rpw + i, r = row_of(sl);
      if (sl >= S || r >= rows) continue;
      Ops::load(partial + (size_t)r * cols, cols, lane, R);
      const float sc = MODE == MTP_RED_INT8TOK ? row_scale(Ops::amax(R)) : 0.f;
      if (two_shot) {
        Ops::wire(d.peer[owner_of(r)] + my_slot, R, r, rows, cols, lane, sc);
      } else {
        for (int q = 0; q < d.ws; ++q) Ops::wire(d.peer[(d.rank + q) % d.ws] + my_slot, R, r, rows, cols, lane, sc);
      }
    }
  };
  if (!two_shot) {
    for (int k = 0; k <= K; ++k) {
      if (k < K) push_round(k);
      stamp();
      if (k >= 1) {
        if (!wait_all(d, site, PH_PUSH, v0 + (uint32_t)(k - 1), all, &abort_sm)) { finish(); return; }
        stamp();
        for (int i = 0; i < rpw; ++i) {
          const int sl = (k - 1) * rpw + i, r = row_of(sl);
          if (sl >= S || r >= rows) continue;
          Ops::reduce(slots, d.ws, r, rows, cols, lane, R);
          Ops::round(R, e.rdt);
          Ops::epilogue(e, R, r, cols, lane);
        }
        stamp();
      }
      if (k < K) signal_rounds(d, site, PH_PUSH, v0 + (uint32_t)k, true, PH_GATHER, 0u, false);
      stamp();
    }
    finish();
    return;
  }
  const char *gath_local = d.peer[d.rank] + d.off_gath[site];
  for (int k = 0; k <= K + 1; ++k) {
    if (k < K) push_round(k);
    stamp();
    if (k >= 1 && k <= K) {
      if (!wait_all(d, site, PH_PUSH, v0 + (uint32_t)(k - 1), all, &abort_sm)) { finish(); return; }
      stamp();
      for (int i = 0; i < rpw; ++i) {
        const int sl = (k - 1) * rpw + i, r = row_of(sl);
        if (sl >= S || r >= rows || owner_of(r) != d.rank) continue;
        Ops::reduce(slots, d.ws, r, rows, cols, lane, R);
        Ops::round(R, e.rdt);
        if constexpr (Ops::EPI == EPI_OUTPROJ) {
          if (sp) {  // the owner runs the epilogue; the normed row is what every rank gathers
            Ops::norm(e, R, r, cols, lane);
            for (int q = 0; q < d.ws; ++q)
              Ops::store_gather(d.peer[(d.rank + q) % d.ws] + d.off_gath[site], R, r, cols, lane, e.out_dtype);
            continue;
          }
        }
        for (int q = 0; q < d.ws; ++q) Ops::store_gather(d.peer[(d.rank + q) % d.ws] + d.off_gath[site], R, r, cols, lane, e.rdt);
      }
      stamp();
    }
    if (k >= 2) {
      if (!wait_all(d, site, PH_GATHER, v0 + (uint32_t)(k - 2), all, &abort_sm)) { finish(); return; }
      stamp();
      for (int i = 0; i < rpw; ++i) {
        const int sl = (k - 2) * rpw + i, r = row_of(sl);
        if (sl >= S || r >= rows) continue;
        if constexpr (Ops::EPI == EPI_OUTPROJ) {
          if (sp) {  // the gathered row is the normed row: copy it out
            Ops::load_gather(gath_local, R, r, cols, lane, e.out_dtype);
            Ops::store_normed(e, R, r, cols, lane);
            continue;
          }
        }
        Ops::load_gather(gath_local, R, r, cols, lane, e.rdt);
        Ops::epilogue(e, R, r, cols, lane);
      }
      stamp();
    }
    if (k <= K) signal_rounds(d, site, PH_PUSH, v0 + (uint32_t)k, k < K, PH_GATHER, v0 + (uint32_t)(k - 1), k >= 1);
    stamp();
  }
  finish();
}

// ----------------------------------------------------------------- standalone quantiser / dequant
__global__ void quantize_rows_kernel(const float *__restrict__ in, int rows, int cols, int ld, float *scales, int8_t *q) {
  MTP_PDL_WAIT();
  MTP_PDL_TRIGGER();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float *row = in + (size_t)warp * ld;
  const float sc = row_scale(row_amax(row, cols, lane));
  if (lane == 0) scales[warp] = sc;
  for (int c = lane; c < cols; c += 32) q[(size_t)warp * cols + c] = (int8_t)quant1(row[c], sc);
}

__global__ void dequant_sum_kernel(const uint8_t *__restrict__ pl, int ws, int rows, int cols, float *out) {
  MTP_PDL_WAIT();
  MTP_PDL_TRIGGER();
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)rows * cols) return;
  const int r = (int)(i / cols);
  const size_t bytes = (size_t)rows * (4 + cols);
  float a = 0.f;
  for (int k = 0; k < ws; ++k) {
    const uint8_t *p = pl + (size_t)k * bytes;
    float s;
    memcpy(&s, p + 4 * (size_t)r, 4);
    a = __fadd_rn(a, __fmul_rn((float)(int8_t)p[4 * (size_t)rows + i], s));
  }
  out[i] = a;
}

// ----------------------------------------------------------------- host
// Fixed row scratch for mtp_allreduce_noalloc: a file-scope device array, so that
// entry point never allocates.  Every GPU that loads the library holds these
// 4 MiB until the process exits.  Host code must not hand the symbol itself to a
// kernel (in host code it only names a host-side stand-in); the device address
// comes from cudaGetSymbolAddress, looked up once per device.  The per-device
// addresses are atomics, so first calls from several host threads do not race.
constexpr size_t NOALLOC_SCRATCH_FLOATS = (size_t)1 << 20;
static __device__ __align__(256) float g_noalloc_scratch[NOALLOC_SCRATCH_FLOATS];
constexpr int MAX_DEVICES = 64;
static std::atomic<float *> g_noalloc_ptr[MAX_DEVICES];

static int current_device(int *dev) {
  if (cudaGetDevice(dev) != cudaSuccess) return fail(MTP_ERR_CUDA, "cudaGetDevice failed");
  if (*dev < 0 || *dev >= MAX_DEVICES) return fail(MTP_ERR_UNSUPPORTED, "device index out of range");
  return MTP_OK;
}

// Device address of g_noalloc_scratch on the current device (set up on first use).
static int noalloc_scratch(float **out) {
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  float *p = g_noalloc_ptr[dev].load(std::memory_order_acquire);
  if (!p) {
    void *q = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&q, g_noalloc_scratch);
    if (e != cudaSuccess)
      return fail(MTP_ERR_CUDA, std::string("cudaGetSymbolAddress(g_noalloc_scratch): ") + cudaGetErrorString(e));
    p = static_cast<float *>(q);
    g_noalloc_ptr[dev].store(p, std::memory_order_release);  // every thread finds the same address
  }
  *out = p;
  return MTP_OK;
}

// Per-warp row scratch of the reduction kernels, one per device.  Grown, never freed: a
// captured CUDA graph may still hold an older pointer.  The first call on a device (eager,
// before any capture) sizes it.  Growth is not thread-safe: one host thread per device.
static float *g_scratch[MAX_DEVICES] = {};
static size_t g_scratch_bytes[MAX_DEVICES] = {};

static float *row_scratch(size_t bytes) {
  int dev = 0;
  if (current_device(&dev)) return nullptr;
  if (bytes > g_scratch_bytes[dev]) {
    float *p = nullptr;
    if (bytes < ((size_t)32 << 20)) bytes = (size_t)32 << 20;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
    g_scratch[dev] = p;
    g_scratch_bytes[dev] = bytes;
  }
  return g_scratch[dev];
}

// Rows wide enough (and outputs aligned) for the 16-column granule layout.  The EPI_XPROJ
// split (dt_low | B|C) keeps the narrow layout: its rows are at most a few hundred values.
static bool wide_ok(int epi, int cols, const EpiOut &e) {
  if (epi == EPI_XPROJ || cols % 16 != 0 || cols < 512 || cols > 3072) return false;
  if (epi == EPI_PLAIN) return aligned16(e.out);
  return aligned16(e.resid) && (!e.bias || aligned16(e.bias)) && (!e.normed || (aligned16(e.normed) && aligned16(e.norm_w)));
}

// Resident CTAs per SM of a pipelined kernel instance (queried once per instance).  With a
// comm context the grid is sized to fill every SM at that occupancy: CTA j only waits for
// CTA j of the other ranks, and CTAs are dispatched in index order, so every launched CTA
// becomes resident once the preceding kernel has drained.
template <class Ops>
static int pipe_occupancy() {
  static int occ = 0;
  if (occ == 0) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, reduce_pipe_kernel<Ops>, WPB * 32, 0) != cudaSuccess || n < 1)
      n = 1;
    occ = n;
  }
  return occ;
}

// Target rounds per reduction launch: MTP_COMM_ROUNDS_X (x_proj site, default 1) and
// MTP_COMM_ROUNDS_OUT (out_proj site and plain reductions, default 1).  Each extra round
// costs a fence and a flag round trip; on B200 one round was fastest at every size measured
// ([32768, 160] and [32768, 2048] at 2 and 4 ranks: +10 to +40% per doubling of rounds).
static int pipe_rounds(int epi) {
  const char *e = getenv(epi == EPI_XPROJ ? "MTP_COMM_ROUNDS_X" : "MTP_COMM_ROUNDS_OUT");
  const int v = e ? atoi(e) : 0;
  return v > 0 && v <= 64 ? v : 1;
}

template <class Ops>
static void launch_pipe(const CommDev &d, bool has_comm, int site, const float *pp, int nr, int cols, bool two_shot,
                        bool sp, const EpiOut &e, int sms, cudaStream_t s) {
  const int Gwant = ceil_div(nr, WPB);
  int cap = has_comm ? sms * pipe_occupancy<Ops>() : sms * 8;
  if (has_comm && cap > G_MAX) cap = G_MAX;
  const int G = Gwant < cap ? Gwant : cap;
  // rows per warp per round from the target number of rounds (each round costs a fence and
  // a flag round trip between the ranks; more rounds overlap more NVLink with HBM work)
  const int slices = ceil_div(nr, G * WPB);
  const int rpw = ceil_div(slices, pipe_rounds(Ops::EPI));
  launch_pdl(reduce_pipe_kernel<Ops>, dim3(G), dim3(WPB * 32), 0, s, d, has_comm, site, pp, nr, cols, two_shot, sp, rpw,
             e);
}

// Wire bytes of one row in `mode`, and of one reduced row in the result dtype.
static size_t wire_row_bytes(int mode, int cols) {
  return mode == MTP_RED_FP32 ? 4 * (size_t)cols : mode == MTP_RED_FP16 ? 2 * (size_t)cols : (size_t)cols + 4;
}
static size_t rdt_row_bytes(int rdt, int cols) { return (rdt == MTP_BF16 ? 2 : 4) * (size_t)cols; }

// Protocol of one reduction launch of nr rows: fewer bytes sent per rank wins; small
// messages stay one-shot (fewer flag rounds).  MTP_COMM_PROTOCOL=oneshot|twoshot overrides.
static bool use_two_shot(int ws, int mode, int nr, int cols, int rdt) {
  if (ws < 2) return false;
  const size_t wire_row = wire_row_bytes(mode, cols), rdt_row = rdt_row_bytes(rdt, cols);
  const double one = (double)(ws - 1) * nr * wire_row;
  const double two = (double)(ws - 1) / ws * nr * (wire_row + rdt_row);
  bool two_shot = two < one && (size_t)nr * wire_row >= ((size_t)1 << 20);
  if (const char *env = getenv("MTP_COMM_PROTOCOL")) {
    if (!strcmp(env, "twoshot")) two_shot = true;
    if (!strcmp(env, "oneshot")) two_shot = false;
  }
  return two_shot;
}

// Bytes one rank sends to its peers for a reduction of [rows, cols] (launches of at most
// max_rows rows): one-shot (ws-1) wire rows per row; two-shot (ws-1)/ws of the wire rows
// to their owners plus (ws-1)/ws of the reduced rows back to every rank.
static double sent_bytes(int ws, int max_rows, int mode, int rows, int cols, int rdt) {
  if (ws < 2) return 0.0;
  double total = 0.0;
  for (int r0 = 0; r0 < rows; r0 += max_rows) {
    const int nr = rows - r0 < max_rows ? rows - r0 : max_rows;
    const double w = (double)nr * wire_row_bytes(mode, cols);
    if (mode >= MTP_RED_INT8TENSOR) {  // one-shot int8 rows (+ the 4-byte maximum of the shared-scale modes)
      total += (double)(ws - 1) * (w + (mode == MTP_RED_INT8TENSOR ? 0.0 : 4.0));
      continue;
    }
    total += use_two_shot(ws, mode, nr, cols, rdt) ? (double)(ws - 1) / ws * (w + (double)nr * rdt_row_bytes(rdt, cols))
                                                   : (double)(ws - 1) * w;
  }
  return total;
}


// ----------------------------------------------------------------- per-tensor-scale int8 reductions
// int8_gather (tp_utils.py:134-142): each rank quantises its whole tensor with one scale
//   max(|x|, 1e-8) / 127, the int8 values are gathered and every rank sums
//   float(q_r) * s_r from zeros in rank order (the per-token arithmetic with one scale per rank);
// int8_sum (:78-100): the scale is shared, max over ranks of max(|x|, 1e-8), / (127 / ws) (integer
//   division), values clamped to +-(127 / ws), summed as integers (exactly, so in any order), times
//   the scale;
// int8_legacy (:45-75): as int8_sum with +-127 (the reference carries int32 on the wire; the sum
//   of int8 values is the same integer).
// tensor_amax_kernel writes per-CTA maxima of |partial|; reduce_scaled_kernel takes their max, and
// for the shared-scale modes CTA 0 pushes it to every rank's slot tail (phase-1 flag of CTA 0) and
// every CTA waits for all ranks' maxima; then one warp per row quantises, pushes the row's int8
// bytes to every rank (one-shot), flags, waits for CTA j of every rank, reduces, rounds and runs the
// site's epilogue.  Receive layout per source rank: [rows x 4 scale bytes | rows x cols int8 | ...
// | max at the slot's last 16 bytes].
__global__ void __launch_bounds__(256) tensor_amax_kernel(const float *__restrict__ x, long n, float *partials) {
  MTP_PDL_WAIT();
  MTP_PDL_TRIGGER();
  __shared__ float wm[8];
  float m = 0.f;
  const long stride = (long)gridDim.x * blockDim.x;
  if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    const long n4 = n / 4;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
      const float4 v = reinterpret_cast<const float4 *>(x)[i];
      m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    for (long i = 4 * n4 + (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) m = fmaxf(m, fabsf(x[i]));
  } else {
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) m = fmaxf(m, fabsf(x[i]));
  }
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) wm[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, wm[w]);
    partials[blockIdx.x] = m;
  }
}

__device__ __forceinline__ int quant_q(float x, float s, float qmax) {
  float r = rintf(__fdiv_rn(x, s));
  r = fminf(fmaxf(r, -qmax), qmax);
  return (int)r;
}

template <int MODE, int EPI>
__global__ void __launch_bounds__(WPB * 32) reduce_scaled_kernel(CommDev d, bool has_comm, int site,
                                                                 const float *__restrict__ partial, int rows, int cols,
                                                                 const float *partials, int G1, float *scratch,
                                                                 EpiOut e) {
  MTP_PDL_WAIT();
  MTP_PDL_TRIGGER();
  __shared__ int abort_sm;
  __shared__ uint32_t epoch_sm;
  __shared__ float amax_sm;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = blockIdx.x, G = gridDim.x;
  if (warp == 0) {
    float m = 0.f;
    for (int i = lane; i < G1; i += 32) m = fmaxf(m, partials[i]);
    m = warp_max(m);
    if (lane == 0) amax_sm = m;
  }
  __syncthreads();
  const float amax = amax_sm;
  const int ws = has_comm ? d.ws : 1;
  const float qmax = MODE == MTP_RED_INT8SUM ? (float)(127 / ws) : 127.0f;
  float *wrow = scratch + (size_t)(j * WPB + warp) * cols;
  if (!has_comm) {
    const float s = MODE == MTP_RED_INT8TENSOR ? row_scale(amax) : __fdiv_rn(fmaxf(amax, 1e-8f), qmax);
    for (int r = j * WPB + warp; r < rows; r += G * WPB) {
      const float *row = partial + (size_t)r * cols;
      for (int c = lane; c < cols; c += 32) {
        const float q = (float)quant_q(row[c], s, qmax);
        wrow[c] = rnd_rdt(MODE == MTP_RED_INT8TENSOR ? __fadd_rn(0.f, __fmul_rn(q, s)) : __fmul_rn(q, s), e.rdt);
      }
      __syncwarp();
      epilogue_row<EPI>(e, wrow, r, cols, lane);
      __syncwarp();
    }
    return;
  }
  uint32_t *ep = reinterpret_cast<uint32_t *>(d.peer[d.rank] + d.off_epoch) + site;
  if (threadIdx.x == 0) {
    abort_sm = 0;
    epoch_sm = *reinterpret_cast<volatile uint32_t *>(ep) + 1u;
  }
  __syncthreads();
  const uint32_t epoch = epoch_sm;
  auto finish = [&]() {
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      unsigned int *done = reinterpret_cast<unsigned int *>(d.peer[d.rank] + d.off_done) + site;
      if (atomicAdd(done, 1u) == (unsigned)G - 1u) {
        *done = 0u;
        *reinterpret_cast<volatile uint32_t *>(ep) = epoch;
        __threadfence();
      }
    }
  };
  const size_t half = (size_t)(epoch & 1u) * d.ws * d.slot_bytes[site];
  const uint32_t all = (1u << d.ws) - 1u;
  const size_t tail = d.slot_bytes[site] - 16;
  float s;
  if (MODE == MTP_RED_INT8TENSOR) {
    s = row_scale(amax);
  } else {
    // the shared scale: every rank's maximum
    if (j == 0 && threadIdx.x < (unsigned)d.ws) {
      *reinterpret_cast<float *>(d.peer[threadIdx.x] + d.off_recv[site] + half + (size_t)d.rank * d.slot_bytes[site] +
                                 tail) = amax;
      __threadfence_system();
      st_release_sys(flag_ptr(d.peer[threadIdx.x], d, site, 1, d.rank, 0), epoch);
    }
    if (threadIdx.x < (unsigned)d.ws) {
      const uint32_t *f = flag_ptr(d.peer[d.rank], d, site, 1, threadIdx.x, 0);
      const unsigned long long t0 = globaltimer_ns();
      uint32_t it = 0;
      while ((int)(ld_acquire_sys(f) - epoch) < 0) {
        if ((++it & 63u) == 0 && globaltimer_ns() - t0 > d.timeout_ns) {
          atomicExch(reinterpret_cast<int *>(d.peer[d.rank] + d.off_status), MTP_ERR_TIMEOUT);
          abort_sm = 1;
          break;
        }
      }
      __threadfence();
    }
    __syncthreads();
    if (abort_sm) { finish(); return; }
    float m = 0.f;
    for (int k = 0; k < d.ws; ++k)
      m = fmaxf(m, __ldcg(reinterpret_cast<const float *>(d.peer[d.rank] + d.off_recv[site] + half +
                                                          (size_t)k * d.slot_bytes[site] + tail)));
    s = __fdiv_rn(fmaxf(m, 1e-8f), qmax);
  }
  // push: every row's int8 values (and, per-tensor, this rank's scale) to every rank
  const size_t my_slot = d.off_recv[site] + half + (size_t)d.rank * d.slot_bytes[site];
  for (int r = j * WPB + warp; r < rows; r += G * WPB) {
    const float *row = partial + (size_t)r * cols;
    for (int q = 0; q < d.ws; ++q) {
      char *dst = d.peer[(d.rank + q) % d.ws] + my_slot;  // stagger destinations across ranks
      if (lane == 0) reinterpret_cast<float *>(dst)[r] = s;
      int8_t *qd = reinterpret_cast<int8_t *>(dst + (size_t)4 * rows + (size_t)r * cols);
      if ((cols & 3) == 0 && (rows & 3) == 0) {
        for (int c = 4 * lane; c < cols; c += 128)
          *reinterpret_cast<uint32_t *>(qd + c) = pack4(quant_q(row[c], s, qmax), quant_q(row[c + 1], s, qmax),
                                                        quant_q(row[c + 2], s, qmax), quant_q(row[c + 3], s, qmax));
      } else {
        for (int c = lane; c < cols; c += 32) qd[c] = (int8_t)quant_q(row[c], s, qmax);
      }
    }
  }
  signal(d, site, 0, epoch, all);
  if (!wait_all(d, site, 0, epoch, all, &abort_sm)) { finish(); return; }
  const char *slots[MAX_WS];
  for (int k = 0; k < d.ws; ++k) slots[k] = d.peer[d.rank] + d.off_recv[site] + half + (size_t)k * d.slot_bytes[site];
  for (int r = j * WPB + warp; r < rows; r += G * WPB) {
    float sk[MAX_WS];
    if (MODE == MTP_RED_INT8TENSOR)
      for (int k = 0; k < d.ws; ++k) sk[k] = __ldcg(reinterpret_cast<const float *>(slots[k]) + r);
    for (int c = lane; c < cols; c += 32) {
      float acc = 0.f;
      if (MODE == MTP_RED_INT8TENSOR) {
        for (int k = 0; k < d.ws; ++k) {
          const float q = (float)__ldcg(reinterpret_cast<const signed char *>(slots[k] + (size_t)4 * rows + (size_t)r * cols + c));
          acc = __fadd_rn(acc, __fmul_rn(q, sk[k]));
        }
      } else {
        int isum = 0;
        for (int k = 0; k < d.ws; ++k)
          isum += (int)__ldcg(reinterpret_cast<const signed char *>(slots[k] + (size_t)4 * rows + (size_t)r * cols + c));
        acc = __fmul_rn((float)isum, s);
      }
      wrow[c] = rnd_rdt(acc, e.rdt);
    }
    __syncwarp();
    epilogue_row<EPI>(e, wrow, r, cols, lane);
    __syncwarp();
  }
  finish();
}

template <int EPI>
static int run_reduce_scaled(mtp_comm *c, int site, int mode, const float *partial, int rows, int cols, EpiOut e,
                             cudaStream_t s) {
  const bool has_comm = c && c->d.ws > 1;
  const int sms = num_sms();
  const int step = has_comm ? c->max_rows : rows;
  for (int r0 = 0; r0 < rows; r0 += step) {
    const int nr = rows - r0 < step ? rows - r0 : step;
    if (has_comm)
      MTP_REQUIRE((size_t)4 * nr + (size_t)nr * cols + 16 <= c->d.slot_bytes[site], "rows exceed the receive slot");
    int G = ceil_div(nr, WPB);
    if (G > sms) G = sms;
    if (G > G_MAX) G = G_MAX;
    const long n = (long)nr * cols;
    int G1 = (int)((n + 4095) / 4096);
    if (G1 > 2 * sms) G1 = 2 * sms;
    if (G1 < 1) G1 = 1;
    float *scr = row_scratch(((size_t)G * WPB * cols + 512) * sizeof(float));
    if (!scr) return fail(MTP_ERR_CUDA, "could not allocate reduction scratch");
    float *partials = scr + (size_t)G * WPB * cols;
    EpiOut ee = e;
    ee.wide = 0;
    if (EPI == EPI_PLAIN) ee.out = e.out + (size_t)r0 * cols;
    if (EPI == EPI_XPROJ) {
      ee.dt_low = (char *)e.dt_low + (size_t)r0 * e.R * (e.dt_dtype == MTP_F32 ? 4 : 2);
      ee.bc = e.bc + (size_t)r0 * (cols - e.R);
    }
    if (EPI == EPI_OUTPROJ) {
      ee.resid = e.resid + (size_t)r0 * cols;
      if (e.normed) ee.normed = (char *)e.normed + (size_t)r0 * cols * (e.out_dtype == MTP_F32 ? 4 : 2);
    }
    const float *pp = partial + (size_t)r0 * cols;
    launch_pdl(tensor_amax_kernel, dim3(G1), dim3(256), 0, s, pp, n, partials);
    int rc = check_launch("tensor_amax");
    if (rc) return rc;
    CommDev d{};
    if (has_comm) d = c->d;
#define MTP_RS(M) launch_pdl(reduce_scaled_kernel<M, EPI>, dim3(G), dim3(WPB * 32), 0, s, d, has_comm, site, pp, nr, cols, \
                             (const float *)partials, G1, scr, ee)
    if (mode == MTP_RED_INT8TENSOR) MTP_RS(MTP_RED_INT8TENSOR);
    else if (mode == MTP_RED_INT8SUM) MTP_RS(MTP_RED_INT8SUM);
    else MTP_RS(MTP_RED_INT8LEGACY);
#undef MTP_RS
    rc = check_launch("reduce_scaled");
    if (rc) return rc;
  }
  return MTP_OK;
}

template <int EPI>
static int run_reduce(mtp_comm *c, int site, int mode, const float *partial, int rows, int cols, EpiOut e,
                      cudaStream_t s) {
  MTP_REQUIRE(partial && rows >= 0 && cols > 0, "bad arguments");
  MTP_REQUIRE(mode >= MTP_RED_FP32 && mode <= MTP_RED_INT8LEGACY, "unknown reduction mode");
  MTP_REQUIRE(aligned16(partial), "partial must be 16-byte aligned");
  if (rows == 0) return MTP_OK;
  const bool has_comm = c && c->d.ws > 1;
  if (has_comm) {
    MTP_REQUIRE(c->opened, "comm context peers not opened");
    MTP_REQUIRE(cols <= c->cols[site], "row width exceeds the context's site width");
  }
  if (mode >= MTP_RED_INT8TENSOR) return run_reduce_scaled<EPI>(c, site, mode, partial, rows, cols, e, s);
  const int sms = num_sms();
  // rows per launch: bounded by the context's slots; each launch is a complete reduction
  const int step = has_comm ? c->max_rows : rows;
  for (int r0 = 0; r0 < rows; r0 += step) {
    const int nr = rows - r0 < step ? rows - r0 : step;
    int G = ceil_div(nr, WPB);
    if (G > sms) G = sms;
    if (G > G_MAX) G = G_MAX;
    const bool capped = has_comm && c->max_ctas > 0;
    if (capped && G > c->max_ctas) G = c->max_ctas;
    float *scr = nullptr;
    if (cols % 4 != 0 || cols > 3072 || capped) {
      scr = row_scratch((size_t)G * WPB * cols * sizeof(float));
      if (!scr) return fail(MTP_ERR_CUDA, "could not allocate reduction scratch");
    }
    EpiOut ee = e;
    // advance outputs by r0 rows
    if (EPI == EPI_PLAIN) ee.out = e.out + (size_t)r0 * cols;
    if (EPI == EPI_XPROJ) {
      ee.dt_low = (char *)e.dt_low + (size_t)r0 * e.R * (e.dt_dtype == MTP_F32 ? 4 : 2);
      ee.bc = e.bc + (size_t)r0 * (cols - e.R);
    }
    if (EPI == EPI_OUTPROJ) {
      ee.resid = e.resid + (size_t)r0 * cols;
      if (e.normed) ee.normed = (char *)e.normed + (size_t)r0 * cols * (e.out_dtype == MTP_F32 ? 4 : 2);
    }
    CommDev d{};
    if (has_comm) d = c->d;
    // sequence-parallel out_proj epilogue: each row's owner rank applies the residual and
    // the next RMSNorm and every rank gathers the normed rows (the residual rows of other
    // owners are then not kept on this rank); needs the normed output and the two-shot
    // protocol, which it implies.  B200, [32768, 2048] int8 / fp16: 338 / 472 us at 2 ranks
    // (one-shot 366 / 634), 409 / 641 us at 4 (two-shot without it 453 / 684).
    // MTP_COMM_SP=0 turns it off.
    bool sp = EPI == EPI_OUTPROJ && has_comm && ee.normed != nullptr && !capped && c->sp_allowed;
    if (sp) {
      const char *env = getenv("MTP_COMM_SP");
      if (env && !strcmp(env, "0")) sp = false;
    }
    const bool two_shot = has_comm && (sp || use_two_shot(c->d.ws, mode, nr, cols, e.rdt));
    const float *pp = partial + (size_t)r0 * cols;
    // wide rows in 16-column granules (16-byte accesses) when the width and the output
    // pointers allow it, else the register-row kernel, else the scratch kernel
    ee.wide = wide_ok(EPI, cols, ee) ? 1 : 0;
    if (!capped && ee.wide) {
      const int nc = (cols + 511) / 512;
#define MTP_PW(M, NCC) launch_pipe<WideOps<M, EPI, NCC>>(d, has_comm, site, pp, nr, cols, two_shot, sp, ee, sms, s)
#define MTP_PW_MODE(NCC)                                    \
  do {                                                      \
    if (mode == MTP_RED_FP32) MTP_PW(MTP_RED_FP32, NCC);      \
    else if (mode == MTP_RED_FP16) MTP_PW(MTP_RED_FP16, NCC); \
    else MTP_PW(MTP_RED_INT8TOK, NCC);                        \
  } while (0)
      switch (nc) {
        case 2: MTP_PW_MODE(2); break;
        case 3: MTP_PW_MODE(3); break;
        case 4: MTP_PW_MODE(4); break;
        case 5: MTP_PW_MODE(5); break;
        default: MTP_PW_MODE(6); break;
      }
#undef MTP_PW_MODE
#undef MTP_PW
      int rc = check_launch("reduce");
      if (rc) return rc;
      continue;
    }
    // register-row kernel when the width allows it
    const int vpl = (cols % 4 != 0 || capped) ? 0 : cols <= 256 ? 2 : cols <= 512 ? 4 : cols <= 1024 ? 8 : cols <= 2048 ? 16 : cols <= 3072 ? 24 : 0;
    if (vpl) {
#define MTP_PV(M, V) launch_pipe<NarrowOps<M, EPI, V>>(d, has_comm, site, pp, nr, cols, two_shot, sp, ee, sms, s)
#define MTP_PV_MODE(V)                                      \
  do {                                                      \
    if (mode == MTP_RED_FP32) MTP_PV(MTP_RED_FP32, V);      \
    else if (mode == MTP_RED_FP16) MTP_PV(MTP_RED_FP16, V); \
    else MTP_PV(MTP_RED_INT8TOK, V);                        \
  } while (0)
      switch (vpl) {
        case 2: MTP_PV_MODE(2); break;
        case 4: MTP_PV_MODE(4); break;
        case 8: MTP_PV_MODE(8); break;
        case 16: MTP_PV_MODE(16); break;
        default: MTP_PV_MODE(24); break;
      }
#undef MTP_PV_MODE
#undef MTP_PV
    } else {
#define MTP_RED_LAUNCH(M) \
  launch_pdl(reduce_kernel<M, EPI>, dim3(G), dim3(WPB * 32), 0, s, d, has_comm, site, pp, nr, cols, two_shot, scr, ee)
      if (mode == MTP_RED_FP32) MTP_RED_LAUNCH(MTP_RED_FP32);
      else if (mode == MTP_RED_FP16) MTP_RED_LAUNCH(MTP_RED_FP16);
      else MTP_RED_LAUNCH(MTP_RED_INT8TOK);
#undef MTP_RED_LAUNCH
    }
    int rc = check_launch("reduce");
    if (rc) return rc;
  }
  return MTP_OK;
}

// ----------------------------------------------------------------- x_proj reduction finished after the GEMM
// Second half of AllReduce #1 when the x_proj GEMM's epilogue wrote the wire rows into
// every rank's receive slots (gemm_tc_xproj_wire): wait (bounded) for the phase-0 flags
// of all Gg GEMM CTAs of every rank, reduce every row over the ranks in rank order (one
// warp per row, the reduction kernels' own arithmetic), round and split into dt_low | B|C;
// the last CTA to leave advances the site's epoch.
template <class Ops>
__global__ void __launch_bounds__(WPB * 32) xproj_finish_kernel(CommDev d, int site, int Gg, int rows, int cols,
                                                                EpiOut e) {
  MTP_PDL_WAIT();
  MTP_PDL_TRIGGER();
  __shared__ int abort_sm;
  __shared__ uint32_t epoch_sm;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = blockIdx.x, G = gridDim.x;
  uint32_t *ep = reinterpret_cast<uint32_t *>(d.peer[d.rank] + d.off_epoch) + site;
  if (threadIdx.x == 0) {
    abort_sm = 0;
    epoch_sm = *reinterpret_cast<volatile uint32_t *>(ep) + 1u;
  }
  __syncthreads();
  const uint32_t epoch = epoch_sm;
  const unsigned long long t0 = globaltimer_ns();  // one bound for all of this CTA's waits
  volatile int *ab = &abort_sm;
  for (int i = threadIdx.x; i < d.ws * Gg && !*ab; i += blockDim.x) {
    const uint32_t *f = flag_ptr(d.peer[d.rank], d, site, 0, i / Gg, i % Gg);
    uint32_t it = 0;
    while ((int)(ld_acquire_sys(f) - epoch) < 0) {
      if ((++it & 63u) == 0 && (*ab || globaltimer_ns() - t0 > d.timeout_ns)) {
        if (!*ab) atomicExch(reinterpret_cast<int *>(d.peer[d.rank] + d.off_status), MTP_ERR_TIMEOUT);
        *ab = 1;
        break;
      }
    }
  }
  __threadfence();
  __syncthreads();
  if (!abort_sm) {
    const size_t half = (size_t)(epoch & 1u) * d.ws * d.slot_bytes[site];
    char *slots[MAX_WS];
    for (int k = 0; k < d.ws; ++k) slots[k] = d.peer[d.rank] + d.off_recv[site] + half + (size_t)k * d.slot_bytes[site];
    typename Ops::Row R;
    for (int r = j * WPB + warp; r < rows; r += G * WPB) {
      Ops::reduce(slots, d.ws, r, rows, cols, lane, R);
      Ops::round(R, e.rdt);
      Ops::epilogue(e, R, r, cols, lane);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    unsigned int *done = reinterpret_cast<unsigned int *>(d.peer[d.rank] + d.off_done) + site;
    if (atomicAdd(done, 1u) == (unsigned)G - 1u) {
      *done = 0u;
      *reinterpret_cast<volatile uint32_t *>(ep) = epoch;
      __threadfence();
    }
  }
}

// ----------------------------------------------------------------- vocabulary-column gather
// Vocabulary-parallel lm_head: rank k holds logits columns [k shard, min(V, (k+1) shard)) of
// every row (shard = vocab_shard()); one launch gives every rank all of them.  Element units
// are U (16 bytes when every row start and shard boundary is 16-byte aligned, else the
// logits element).  CTA j handles units [j per, (j+1) per) of the [rows, shard] block, the
// same range on every rank: it copies its own columns into `out`, pushes them to every
// peer's receive slot of `site` (half by epoch parity, as the reductions), raises its
// flag, waits (bounded) for CTA j of every rank and copies the peers' columns out.  The
// epoch / parity protocol is the reductions' own, so the launch can follow or precede a
// reduction on the same site.
template <typename U>
__global__ void __launch_bounds__(256) gather_cols_kernel(CommDev d, int site, U *out, long ldo, int rows,
                                                          int shard_u, int total_u) {
  MTP_PDL_WAIT();
  MTP_PDL_TRIGGER();
  __shared__ int abort_sm;
  __shared__ uint32_t epoch_sm;
  const int j = blockIdx.x, G = gridDim.x;
  uint32_t *ep = reinterpret_cast<uint32_t *>(d.peer[d.rank] + d.off_epoch) + site;
  if (threadIdx.x == 0) {
    abort_sm = 0;
    epoch_sm = *reinterpret_cast<volatile uint32_t *>(ep) + 1u;
  }
  __syncthreads();
  const uint32_t epoch = epoch_sm;
  const size_t half = (size_t)(epoch & 1u) * d.ws * d.slot_bytes[site];
  const uint32_t all = (1u << d.ws) - 1u;
  const long n = (long)rows * shard_u;
  const long per = (n + G - 1) / G, lo = (long)j * per, hi = lo + per < n ? lo + per : n;
  auto cols_of = [&](int k) {
    const int c = total_u - k * shard_u;
    return c < shard_u ? c : shard_u;
  };
  const int mine = cols_of(d.rank);
  const long col0 = (long)d.rank * shard_u;
  for (int q = 1; q < d.ws; ++q) {
    const int dst = (d.rank + q) % d.ws;  // stagger destinations across ranks
    U *slot = reinterpret_cast<U *>(d.peer[dst] + d.off_recv[site] + half + (size_t)d.rank * d.slot_bytes[site]);
    for (long i = lo + threadIdx.x; i < hi; i += blockDim.x) {
      const long r = i / shard_u;
      const int c = (int)(i - r * shard_u);
      if (c < mine) slot[i] = out[r * ldo + col0 + c];
    }
  }
  signal(d, site, 0, epoch, all);
  bool ok = wait_all(d, site, 0, epoch, all, &abort_sm);
  if (ok) {
    for (int q = 1; q < d.ws; ++q) {
      const int src = (d.rank + q) % d.ws;
      const U *slot = reinterpret_cast<const U *>(d.peer[d.rank] + d.off_recv[site] + half + (size_t)src * d.slot_bytes[site]);
      const int cs = cols_of(src);
      const long c0 = (long)src * shard_u;
      for (long i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const long r = i / shard_u;
        const int c = (int)(i - r * shard_u);
        if (c < cs) out[r * ldo + c0 + c] = __ldcg(slot + i);
      }
    }
  }
  // the last CTA to leave publishes the epoch for the next call
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    unsigned int *done = reinterpret_cast<unsigned int *>(d.peer[d.rank] + d.off_done) + site;
    if (atomicAdd(done, 1u) == (unsigned)G - 1u) {
      *done = 0u;
      *reinterpret_cast<volatile uint32_t *>(ep) = epoch;
      __threadfence();
    }
  }
}

// Columns of each rank in the vocabulary-parallel lm_head: ceil(V / ws) rounded up to a
// multiple of 8 (16-byte boundaries for 2-byte logits), the last rank the remainder.
int vocab_shard(int V, int ws) {
  const int s = (V + ws - 1) / ws;
  return (s + 7) / 8 * 8;
}

int gemm_cols_as_full(const void *A, const void *B, void *C, int M, int N_full, int col0, int cols, int K, int lda,
                      int ldb, int ldc, int dtype, cudaStream_t s);
bool gemm_tc_eligible(const void *A, const void *B, int M, int N, int K, int lda, int ldb);

}  // namespace mtp

using namespace mtp;

extern "C" {

int mtp_comm_create(int rank, int world_size, int max_rows, int cols_x, int cols_out, double timeout_s, mtp_comm **out) {
  MTP_REQUIRE(out, "null out");
  MTP_REQUIRE(world_size >= 1 && world_size <= MAX_WS && rank >= 0 && rank < world_size, "bad rank / world size");
  MTP_REQUIRE(max_rows > 0 && cols_x > 0 && cols_out > 0, "bad sizes");
  mtp_comm *c = new mtp_comm();
  c->max_rows = max_rows;
  c->cols[0] = cols_x;
  c->cols[1] = cols_out;
  auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
  size_t off = 0;
  c->d.off_flags = off;
  off = al(off + sizeof(uint32_t) * 2 * NPHASE * MAX_WS * G_MAX);
  c->d.off_epoch = off;
  off = al(off + sizeof(uint32_t) * 2);
  c->d.off_done = off;
  off = al(off + sizeof(uint32_t) * 2);
  c->d.off_status = off;
  off = al(off + 256);
  for (int s = 0; s < 2; ++s) {
    c->d.slot_bytes[s] = al((size_t)max_rows * (4 * (size_t)c->cols[s] + 16));
    c->d.off_recv[s] = off;
    off = al(off + c->d.slot_bytes[s] * world_size * 2);  // two halves, by epoch parity
    c->d.off_gath[s] = off;
    off = al(off + (size_t)max_rows * c->cols[s] * 4);
  }
  c->total = off;
  if (cudaMalloc(&c->base, c->total) != cudaSuccess) {
    delete c;
    return fail(MTP_ERR_CUDA, "cudaMalloc of the comm buffers failed");
  }
  cudaMemset(c->base, 0, c->d.off_recv[0]);
  c->d.rank = rank;
  c->d.ws = world_size;
  c->d.timeout_ns = (unsigned long long)(timeout_s * 1e9);
  for (int k = 0; k < MAX_WS; ++k) c->d.peer[k] = nullptr;
  c->d.peer[rank] = c->base;
  if (world_size > 1 && cudaIpcGetMemHandle(&c->handle, c->base) != cudaSuccess) {
    cudaFree(c->base);
    delete c;
    return fail(MTP_ERR_CUDA, "cudaIpcGetMemHandle failed");
  }
  c->opened = world_size == 1;
  if (cudaDeviceSynchronize() != cudaSuccess) return fail(MTP_ERR_CUDA, "comm init sync failed");
  *out = c;
  return MTP_OK;
}

int mtp_comm_ipc_handle(mtp_comm *c, void *handle64) {
  MTP_REQUIRE(c && handle64, "null argument");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  memcpy(handle64, &c->handle, 64);
  return MTP_OK;
}

int mtp_comm_open_peers(mtp_comm *c, const void *handles) {
  MTP_REQUIRE(c && handles, "null argument");
  for (int k = 0; k < c->d.ws; ++k) {
    if (k == c->d.rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, (const char *)handles + 64 * k, 64);
    void *p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return fail(MTP_ERR_CUDA, std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
    c->d.peer[k] = (char *)p;
  }
  c->opened = true;
  return MTP_OK;
}

int mtp_comm_destroy(mtp_comm *c) {
  if (!c) return MTP_OK;
  cudaDeviceSynchronize();
  if (c->d.trace) cudaFree(c->d.trace);
  for (int k = 0; k < c->d.ws; ++k)
    if (k != c->d.rank && c->d.peer[k]) cudaIpcCloseMemHandle(c->d.peer[k]);
  if (c->base) cudaFree(c->base);
  delete c;
  return MTP_OK;
}

int mtp_comm_status(mtp_comm *c, int *status) {
  MTP_REQUIRE(c && status, "null argument");
  if (cudaMemcpy(status, c->base + c->d.off_status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return fail(MTP_ERR_CUDA, "reading the comm status failed");
  return MTP_OK;
}

int mtp_comm_set_trace(mtp_comm *c, int records) {
  MTP_REQUIRE(c && records >= 0, "bad arguments");
  if (c->d.trace) {
    cudaDeviceSynchronize();
    cudaFree(c->d.trace);
    c->d.trace = nullptr;
    c->d.trace_count = nullptr;
    c->d.trace_cap = 0;
  }
  if (records == 0) return MTP_OK;
  const size_t bytes = (size_t)records * TRACE_WORDS * 8 + 16;
  void *p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return fail(MTP_ERR_CUDA, "cudaMalloc of the trace buffer failed");
  cudaMemset(p, 0, bytes);
  c->d.trace = static_cast<unsigned long long *>(p);
  c->d.trace_count = reinterpret_cast<unsigned int *>(static_cast<char *>(p) + (size_t)records * TRACE_WORDS * 8);
  c->d.trace_cap = records;
  return cudaDeviceSynchronize() == cudaSuccess ? MTP_OK : fail(MTP_ERR_CUDA, "trace set-up failed");
}

int mtp_comm_read_trace(mtp_comm *c, uint64_t *out, int capacity, int *n_records) {
  MTP_REQUIRE(c && out && n_records && c->d.trace, "tracing is off or bad arguments");
  unsigned int cnt[2] = {0, 0};
  if (cudaMemcpy(cnt, c->d.trace_count, 8, cudaMemcpyDeviceToHost) != cudaSuccess) return fail(MTP_ERR_CUDA, "read trace");
  int n = (int)(cnt[0] < (unsigned)c->d.trace_cap ? cnt[0] : (unsigned)c->d.trace_cap);
  if (n * TRACE_WORDS > capacity) n = capacity / TRACE_WORDS;
  if (n > 0 && cudaMemcpy(out, c->d.trace, (size_t)n * TRACE_WORDS * 8, cudaMemcpyDeviceToHost) != cudaSuccess)
    return fail(MTP_ERR_CUDA, "read trace");
  *n_records = n;
  return MTP_OK;
}

int mtp_comm_set_max_ctas(mtp_comm *c, int max_ctas) {
  MTP_REQUIRE(c && max_ctas >= 0, "bad arguments");
  c->max_ctas = max_ctas;
  return MTP_OK;
}

int mtp_comm_set_sequence_parallel(mtp_comm *c, int on) {
  MTP_REQUIRE(c, "null argument");
  c->sp_allowed = on != 0;
  return MTP_OK;
}

int mtp_comm_reset_state(mtp_comm *c) {
  MTP_REQUIRE(c, "null argument");
  // flags, epochs, exit counters and the status word (everything before the receive slots)
  if (cudaDeviceSynchronize() != cudaSuccess || cudaMemset(c->base, 0, c->d.off_recv[0]) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess)
    return fail(MTP_ERR_CUDA, "reset of the comm state failed");
  return MTP_OK;
}

int mtp_comm_reset_status(mtp_comm *c) {
  MTP_REQUIRE(c, "null argument");
  if (cudaMemset(c->base + c->d.off_status, 0, sizeof(int)) != cudaSuccess) return fail(MTP_ERR_CUDA, "reset status");
  return MTP_OK;
}

int mtp_comm_sent_bytes(mtp_comm *c, int mode, int rows, int cols, int rdt, double *bytes) {
  MTP_REQUIRE(bytes && rows >= 0 && cols > 0, "bad arguments");
  *bytes = (c && c->d.ws > 1) ? sent_bytes(c->d.ws, c->max_rows, mode, rows, cols, rdt) : 0.0;
  return MTP_OK;
}

int mtp_reduce_xproj(mtp_comm *c, int mode, const float *partial, int rows, int R, int N2, void *dt_low, int dt_dtype,
                     float *bc, void *stream) {
  MTP_REQUIRE(dt_low && bc && R > 0 && N2 > 0, "bad arguments");
  MTP_REQUIRE(dt_dtype == MTP_F32 || dt_dtype == MTP_BF16, "dt_low must be F32 or BF16");
  EpiOut e{};
  e.dt_low = dt_low;
  e.bc = bc;
  e.R = R;
  e.dt_dtype = dt_dtype;
  e.rdt = dt_dtype;
  return run_reduce<EPI_XPROJ>(c, 0, mode, partial, rows, R + N2, e, (cudaStream_t)stream);
}

int mtp_reduce_outproj(mtp_comm *c, int mode, const float *partial, int rows, int D, const void *bias, float *resid,
                       const void *norm_w, float eps, void *normed, int out_dtype, void *stream) {
  MTP_REQUIRE(resid && D > 0, "bad arguments");
  MTP_REQUIRE(!normed || norm_w, "normed output needs norm weights");
  MTP_REQUIRE(out_dtype == MTP_F32 || out_dtype == MTP_BF16, "out dtype must be F32 or BF16");
  EpiOut e{};
  e.bias = bias;
  e.resid = resid;
  e.norm_w = norm_w;
  e.normed = normed;
  e.eps = eps;
  e.out_dtype = out_dtype;
  e.rdt = out_dtype;
  return run_reduce<EPI_OUTPROJ>(c, 1, mode, partial, rows, D, e, (cudaStream_t)stream);
}

int mtp_allreduce(mtp_comm *c, int site, int mode, const float *in, float *out, int rows, int cols, void *stream) {
  MTP_REQUIRE(out && (site == 0 || site == 1), "bad arguments");
  EpiOut e{};
  e.out = out;
  e.rdt = MTP_F32;
  return run_reduce<EPI_PLAIN>(c, site, mode, in, rows, cols, e, (cudaStream_t)stream);
}

int mtp_allreduce_noalloc(int mode, const float *in, float *out, int rows, int cols, void *stream) {
  MTP_REQUIRE(in && out && rows >= 0 && cols > 0, "bad arguments");
  MTP_REQUIRE(mode == MTP_RED_FP32 || mode == MTP_RED_FP16 || mode == MTP_RED_INT8TOK, "unknown reduction mode");
  MTP_REQUIRE((size_t)cols <= NOALLOC_SCRATCH_FLOATS / WPB,
              "mtp_allreduce_noalloc: cols exceeds the fixed scratch (at most 131072 values per row)");
  if (rows == 0) return MTP_OK;
  float *scr = nullptr;
  const int rc = noalloc_scratch(&scr);
  if (rc) return rc;
  // rows in flight are bounded by the fixed scratch: G CTAs x WPB warps x cols floats
  int G = ceil_div(rows, WPB);
  const int sms = num_sms();
  if (G > sms) G = sms;
  const int cap = (int)(NOALLOC_SCRATCH_FLOATS / ((size_t)WPB * cols));
  if (G > cap) G = cap;
  EpiOut e{};
  e.out = out;
  CommDev d{};
  cudaStream_t s = (cudaStream_t)stream;
  if (mode == MTP_RED_FP32) launch_pdl(reduce_kernel<MTP_RED_FP32, EPI_PLAIN>, dim3(G), dim3(WPB * 32), 0, s, d, false, 1, in, rows, cols, false, scr, e);
  else if (mode == MTP_RED_FP16) launch_pdl(reduce_kernel<MTP_RED_FP16, EPI_PLAIN>, dim3(G), dim3(WPB * 32), 0, s, d, false, 1, in, rows, cols, false, scr, e);
  else launch_pdl(reduce_kernel<MTP_RED_INT8TOK, EPI_PLAIN>, dim3(G), dim3(WPB * 32), 0, s, d, false, 1, in, rows, cols, false, scr, e);
  return check_launch("allreduce_noalloc");
}

int mtp_quantize_rows_int8(const float *in, int rows, int cols, int ld, float *scales, int8_t *q, void *stream) {
  MTP_REQUIRE(in && scales && q && rows >= 0 && cols > 0 && ld >= cols, "bad arguments");
  if (rows == 0) return MTP_OK;
  launch_pdl(quantize_rows_kernel, dim3(ceil_div(rows, 8)), dim3(256), 0, (cudaStream_t)stream, in, rows, cols, ld, scales, q);
  return check_launch("quantize_rows_int8");
}

int mtp_dequant_sum(const uint8_t *payloads, int ws, int rows, int cols, float *out, void *stream) {
  MTP_REQUIRE(payloads && out && ws >= 1 && rows >= 0 && cols > 0, "bad arguments");
  if (rows == 0) return MTP_OK;
  const size_t n = (size_t)rows * cols;
  launch_pdl(dequant_sum_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, (cudaStream_t)stream, payloads, ws, rows, cols, out);
  return check_launch("dequant_sum");
}

int mtp_xproj_fused(mtp_comm *c, int mode, const void *xc, int ld_xc, const void *w, int ld_w, int ab_dtype, int rows,
                    int N, int K, int R, float *partial, void *dt_low, int dt_dtype, float *bc, void *stream) {
  MTP_REQUIRE(xc && w && dt_low && bc && rows >= 0 && N > R && R > 0 && K > 0, "bad arguments");
  MTP_REQUIRE(mode == MTP_RED_FP32 || mode == MTP_RED_FP16 || mode == MTP_RED_INT8TOK, "unknown reduction mode");
  MTP_REQUIRE(dt_dtype == MTP_F32 || dt_dtype == MTP_BF16, "dt_low must be F32 or BF16");
  if (rows == 0) return MTP_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const bool has_comm = c && c->d.ws > 1;
  // default: the fused form at world sizes 1 and 2 (B200, 1.4b 32 x 1024: 79 vs 105 us per
  // layer at 1 rank, 110 vs ~100 at 2); from 3 ranks on, its one-shot push sends every row to
  // every rank, more than the reduction kernel's two-shot protocol moves, so the kernel pair
  // stays the default there.  MTP_XPROJ_FUSED=1 forces it at any world size, 0 turns it off.
  // Also only with at least half an SM-wave of 128-row tiles: the epilogue form keeps whole
  // rows in one N tile, so short inputs would run on a few CTAs where the kernel pair's GEMM
  // narrows its N tile to fill the SMs.
  const char *fenv = getenv("MTP_XPROJ_FUSED");
  const bool fused_on = fenv ? fenv[0] == '1'
                             : ((!has_comm || c->d.ws <= 2) && (long)ceil_div(rows, 128) * 2 >= num_sms());
  MTP_REQUIRE(ab_dtype == MTP_F32 || ab_dtype == MTP_BF16, "xc / w must be F32 or BF16");
  const bool fused = fused_on && ab_dtype == MTP_BF16 && gemm_tc_eligible(xc, w, rows, N, K, ld_xc, ld_w) && N % 16 == 0 && N <= 192 &&
                     R % 16 == 0 && aligned16(dt_low) && aligned16(bc) &&
                     (!has_comm || (mode == MTP_RED_INT8TOK && c->opened && N <= c->cols[0] && rows <= c->max_rows &&
                                    c->max_ctas == 0));
  if (!fused) {  // the GEMM into the fp32 partial, then the reduction kernel
    MTP_REQUIRE(partial, "this x_proj shape needs the fp32 partial buffer");
    int rc = mtp_gemm(xc, w, partial, rows, N, K, ld_xc, ld_w, N, ab_dtype, MTP_F32, MTP_EPI_STORE, nullptr, 0, stream);
    if (rc) return rc;
    return mtp_reduce_xproj(c, mode, partial, rows, R, N - R, dt_low, dt_dtype, bc, stream);
  }
  XprojWire x{};
  x.wmode = mode;
  x.rdt = dt_dtype;
  x.R = R;
  x.dt_dtype = dt_dtype;
  x.ws = has_comm ? c->d.ws : 1;
  x.rank = has_comm ? c->d.rank : 0;
  x.dt_low = dt_low;
  x.bc = bc;
  const int site = 0;
  if (has_comm) {
    const CommDev &d = c->d;
    for (int k = 0; k < d.ws; ++k) {
      x.wslot[k] = d.peer[k] + d.off_recv[site] + (size_t)d.rank * d.slot_bytes[site];
      x.wflag[k] = reinterpret_cast<uint32_t *>(d.peer[k] + d.off_flags) +
                   ((size_t)(site * NPHASE + 0) * MAX_WS + d.rank) * G_MAX;
    }
    x.whalf = (unsigned long long)d.ws * d.slot_bytes[site];
    x.wepoch = reinterpret_cast<const uint32_t *>(d.peer[d.rank] + d.off_epoch) + site;
  }
  int Gg = 0;
  int rc = gemm_tc_xproj_wire(xc, w, rows, N, K, ld_xc, ld_w, x, &Gg, s);
  if (rc || !has_comm) return rc;
  MTP_REQUIRE(Gg <= G_MAX, "GEMM grid exceeds the flag slots");
  EpiOut e{};
  e.dt_low = dt_low;
  e.bc = bc;
  e.R = R;
  e.dt_dtype = dt_dtype;
  e.rdt = dt_dtype;
  const int sms = num_sms();
  int G = ceil_div(rows, WPB);
  if (G > 2 * sms) G = 2 * sms;
  const int vpl = N <= 128 ? 1 : 2;  // 4 values per lane per chunk: 128 columns per chunk
  CommDev d = c->d;
#define MTP_XF(M, V) launch_pdl(xproj_finish_kernel<NarrowOps<M, EPI_XPROJ, V>>, dim3(G), dim3(WPB * 32), 0, s, d, site, Gg, rows, N, e)
#define MTP_XF_MODE(V)                                      \
  do {                                                      \
    if (mode == MTP_RED_FP32) MTP_XF(MTP_RED_FP32, V);      \
    else if (mode == MTP_RED_FP16) MTP_XF(MTP_RED_FP16, V); \
    else MTP_XF(MTP_RED_INT8TOK, V);                        \
  } while (0)
  if (vpl == 1) MTP_XF_MODE(1);
  else MTP_XF_MODE(2);
#undef MTP_XF_MODE
#undef MTP_XF
  return check_launch("xproj_finish");
}

int mtp_vocab_shard(int V, int world_size, int rank, int *col0, int *cols) {
  MTP_REQUIRE(V > 0 && world_size >= 1 && rank >= 0 && rank < world_size && col0 && cols, "bad arguments");
  const int sh = vocab_shard(V, world_size);
  MTP_REQUIRE((long)sh * (world_size - 1) < V, "vocabulary too small for the rank count");
  *col0 = sh * rank;
  *cols = V - sh * rank < sh ? V - sh * rank : sh;
  return MTP_OK;
}

int mtp_lm_head_vocab_parallel(mtp_comm *c, const void *normed, int rows, int K, int ld_normed, const void *emb, int V,
                               int ld_emb, int dtype, void *out, int ld_out, void *stream) {
  MTP_REQUIRE(normed && emb && out && rows >= 0 && K > 0 && V > 0, "bad arguments");
  MTP_REQUIRE(dtype == MTP_F32 || dtype == MTP_BF16, "dtype must be F32 or BF16");
  MTP_REQUIRE(ld_normed >= K && ld_emb >= K && ld_out >= V, "leading dimensions too small");
  if (rows == 0) return MTP_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const bool has_comm = c && c->d.ws > 1;
  if (!has_comm) return mtp_gemm(normed, emb, out, rows, V, K, ld_normed, ld_emb, ld_out, dtype, dtype, MTP_EPI_STORE,
                                 nullptr, 0, stream);
  MTP_REQUIRE(c->opened, "comm context peers not opened");
  const int ws = c->d.ws, rank = c->d.rank, site = 1;
  int col0 = 0, cols = 0;
  int rc = mtp_vocab_shard(V, ws, rank, &col0, &cols);
  if (rc) return rc;
  const int sh = vocab_shard(V, ws);
  const size_t es = dtype == MTP_F32 ? 4 : 2;
  MTP_REQUIRE((size_t)rows * sh * es <= c->d.slot_bytes[site], "rows x vocabulary shard exceed the receive slot");
  rc = gemm_cols_as_full(normed, emb, out, rows, V, col0, cols, K, ld_normed, ld_emb, ld_out, dtype, s);
  if (rc) return rc;
  const bool v16 = aligned16(out) && ((size_t)ld_out * es) % 16 == 0 && ((size_t)sh * es) % 16 == 0 &&
                   ((size_t)V * es) % 16 == 0;
  const int upe = v16 ? (int)(16 / es) : 1;  // elements per unit
  const int shard_u = sh / upe, total_u = V / upe;
  const long n = (long)rows * shard_u;
  int G = (int)((n + 1023) / 1024);
  const int gmax = 2 * num_sms() < G_MAX ? 2 * num_sms() : G_MAX;
  if (G > gmax) G = gmax;
  if (G < 1) G = 1;
  CommDev d = c->d;
  if (v16)
    launch_pdl(gather_cols_kernel<uint4>, dim3(G), dim3(256), 0, s, d, site, (uint4 *)out, (long)(ld_out / upe), rows,
               shard_u, total_u);
  else if (es == 4)
    launch_pdl(gather_cols_kernel<uint32_t>, dim3(G), dim3(256), 0, s, d, site, (uint32_t *)out, (long)ld_out, rows,
               shard_u, total_u);
  else
    launch_pdl(gather_cols_kernel<uint16_t>, dim3(G), dim3(256), 0, s, d, site, (uint16_t *)out, (long)ld_out, rows,
               shard_u, total_u);
  return check_launch("gather_cols");
}

}  // extern "C"
