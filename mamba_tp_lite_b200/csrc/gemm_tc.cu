// tcgen05 / TMEM tensor-core GEMM for sm_100a:  C[M,N] = A[M,K] . B[N,K]^T  (bf16 in, fp32 accumulate).
//
// Persistent, warp-specialised CTA of 6 warps (one CTA per SM):
//   warp 0      one lane issues TMA tile loads (A 128x64, B bn x64, 128-byte swizzle) into a
//               4-stage shared-memory ring, completion tracked by mbarrier transaction counts;
//   warp 1      allocates 512 TMEM columns (two 128 x bn fp32 accumulators) and one lane issues
//               tcgen05.mma (kind::f16, M=128, N=bn, K=16 per instruction), releasing ring slots
//               and signalling finished accumulators with tcgen05.commit;
//   warps 2-13  epilogue: three warps per TMEM lane quarter, alternating 16-column chunks;
//               tcgen05.ld 32 lanes x 16 columns, fused epilogue op, then the 32 x 16 chunk is
//               staged in shared memory and written by a TMA store (or, with unaligned C,
//               stored directly); overlaps the next tile's MMAs thanks to the second accumulator.
// Every mbarrier wait is bounded (globaltimer); on expiry the CTA records MTP_ERR_TIMEOUT in a
// device word, drains its in-flight copies and MMAs with bounded waits, frees TMEM and returns.
#include <cuda.h>
#include "common.cuh"
#include "tc_common.cuh"
#include "wire.cuh"

namespace mtp {
namespace tc {

constexpr int BM = 128, BK = 64, BN_MAX = 256, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN_MAX * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int NUM_EPI_WARPS = 12;  // 3 per TMEM lane quarter
constexpr int EPI_PARTS = NUM_EPI_WARPS / 4;  // warps sharing a lane quarter split its 16-column chunks
constexpr int NUM_THREADS = 64 + 32 * NUM_EPI_WARPS;
constexpr uint32_t TMEM_COLS = 512;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align slack*/ + 256 /*barriers*/;
// Epilogue staging for TMA stores: per epilogue warp two 32-row x 16-column bf16 chunks
// (double buffer) or one fp32 chunk, 2 KB, after the barrier block.
constexpr int STAGE_C_BYTES = 2048;
constexpr int SMEM_BYTES_TMA_STORE = SMEM_BYTES + NUM_EPI_WARPS * STAGE_C_BYTES;

struct Params {
  void *C;
  const void *bias;
  int *err;
  unsigned long long timeout_ns;
  int M, N, K, ldc;
  int c_dtype, epi, bias_dtype;
  int bn, tiles_m, tiles_n, num_tiles, group_m;
  uint32_t idesc;
  int vec_ok;     // 16-byte vector stores allowed
  int tma_store;  // the epilogue stages 32 x 16 chunks in shared memory and writes them with TMA
  int wire;       // x_proj reduction epilogue (one N tile holds whole rows; C is not written)
  XprojWire x;
};

__device__ __forceinline__ void tile_coords(const Params &p, int t, int &mt, int &nt) {
  const int gsize = p.group_m * p.tiles_n;
  const int g = t / gsize;
  const int first_m = g * p.group_m;
  const int gm = min(p.tiles_m - first_m, p.group_m);
  const int r = t - g * gsize;
  mt = first_m + r % gm;
  nt = r / gm;
}

__device__ __forceinline__ float load_bias(const Params &p, int n) {
  return p.bias_dtype == MTP_F32 ? ((const float *)p.bias)[n] : __bfloat162float(((const __nv_bfloat16 *)p.bias)[n]);
}

// 16 bias values for columns [n0, n0+16): vector loads when the whole group is in range.
__device__ __forceinline__ void load_bias16(const Params &p, int n0, float (&b)[16]) {
  if (p.bias_dtype == MTP_F32 && n0 + 16 <= p.N && (reinterpret_cast<uintptr_t>((const float *)p.bias + n0) & 15) == 0) {
    const float4 *bp = reinterpret_cast<const float4 *>((const float *)p.bias + n0);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 v = __ldg(bp + i);
      b[4 * i] = v.x; b[4 * i + 1] = v.y; b[4 * i + 2] = v.z; b[4 * i + 3] = v.w;
    }
  } else if (p.bias_dtype == MTP_BF16 && n0 + 16 <= p.N &&
             (reinterpret_cast<uintptr_t>((const __nv_bfloat16 *)p.bias + n0) & 15) == 0) {
    const uint4 *bp = reinterpret_cast<const uint4 *>((const __nv_bfloat16 *)p.bias + n0);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint4 u = __ldg(bp + i);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[k]));
        b[8 * i + 2 * k] = f.x;
        b[8 * i + 2 * k + 1] = f.y;
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) b[i] = (n0 + i < p.N) ? load_bias(p, n0 + i) : 0.f;
  }
}

// Apply the epilogue to 16 accumulator columns [n0, n0+16) of row `row` and store.
__device__ __forceinline__ void epilogue_op(const Params &p, float (&v)[16], const float (&b)[16]);

__device__ __forceinline__ void epilogue_store(const Params &p, int row, int n0, float (&v)[16], const float (&b)[16]) {
  epilogue_op(p, v, b);
  if (row >= p.M) return;
  const bool full = p.vec_ok && (n0 + 16 <= p.N);
  if (p.c_dtype == MTP_F32) {
    float *c = (float *)p.C + (size_t)row * p.ldc + n0;
    if (full) {
#pragma unroll
      for (int i = 0; i < 16; i += 4) *(float4 *)(c + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (n0 + i < p.N) c[i] = v[i];
    }
  } else {
    __nv_bfloat16 *c = (__nv_bfloat16 *)p.C + (size_t)row * p.ldc + n0;
    if (full) {
      uint32_t w[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        w[i] = *reinterpret_cast<uint32_t *>(&h2);
      }
      *(uint4 *)c = make_uint4(w[0], w[1], w[2], w[3]);
      *(uint4 *)(c + 8) = make_uint4(w[4], w[5], w[6], w[7]);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (n0 + i < p.N) c[i] = __float2bfloat16_rn(v[i]);
    }
  }
}

// The epilogue op (bias / softplus) without the store.  A bf16 output is rounded to 8
// bits of mantissa, so its softplus takes the two-MUFU form.
__device__ __forceinline__ void epilogue_op(const Params &p, float (&v)[16], const float (&b)[16]) {
  if (p.epi == MTP_EPI_BIAS_SOFTPLUS) {
    if (p.c_dtype == MTP_BF16) {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = softplus_bf16out(v[i] + b[i]);
      return;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = softplus_fast(v[i] + b[i]);
  } else if (p.epi == MTP_EPI_BIAS) {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] += b[i];
  }
}

// Row `lane` of a 32 x 16 staging chunk (row-major, 16 values per row) from registers.
__device__ __forceinline__ void stage_row(const Params &p, unsigned char *buf, int lane, const float (&v)[16]) {
  if (p.c_dtype == MTP_F32) {
    float4 *o = reinterpret_cast<float4 *>(buf + (size_t)lane * 64);
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  } else {
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t *>(&h2);
    }
    uint4 *o = reinterpret_cast<uint4 *>(buf + (size_t)lane * 32);
    o[0] = make_uint4(w[0], w[1], w[2], w[3]);
    o[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
}

// TMA store of a staged 32 x 16 chunk to C[m0 .. m0+31][n0 .. n0+15] (rows and columns
// outside C are clipped by the copy); one bulk group per chunk.
__device__ __forceinline__ void tma_store_chunk(const CUtensorMap *tm, uint32_t src, int n0, int m0) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tm), "r"(src),
               "r"(n0), "r"(m0)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// x_proj reduction epilogue at world size 1 for 16 accumulator columns [n0, n0+16) of row
// `row`: the wire format's round trip (as the reduction kernels' world-size-1 path),
// rounded to the reduction's return dtype, split into dt_low (columns < R) and B|C.
__device__ __forceinline__ void wire_chunk_local(const Params &p, int row, int n0, const float (&v)[16], float s) {
  float o[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float x = p.x.wmode == MTP_RED_INT8TOK ? dq1(v[i], s) : p.x.wmode == MTP_RED_FP16 ? h1(v[i]) : v[i];
    o[i] = rnd_rdt(x, p.x.rdt);
  }
  if (n0 < p.x.R) {
    if (p.x.dt_dtype == MTP_F32) {
      float4 *d = reinterpret_cast<float4 *>((float *)p.x.dt_low + (size_t)row * p.x.R + n0);
#pragma unroll
      for (int i = 0; i < 4; ++i) d[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
    } else {
      uint32_t w[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        __nv_bfloat162 h2 = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
        w[i] = *reinterpret_cast<uint32_t *>(&h2);
      }
      uint4 *d = reinterpret_cast<uint4 *>((__nv_bfloat16 *)p.x.dt_low + (size_t)row * p.x.R + n0);
      d[0] = make_uint4(w[0], w[1], w[2], w[3]);
      d[1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
  } else {
    float4 *d = reinterpret_cast<float4 *>(p.x.bc + (size_t)row * (p.N - p.x.R) + (n0 - p.x.R));
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
  }
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const Params p) {
  extern __shared__ __align__(1024) unsigned char smem_dyn[];
  const uint32_t raw = smem_u32(smem_dyn);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char *gbase = smem_dyn + (base - raw);
  // barrier block after the stage ring
  const uint32_t bar0 = base + STAGES * STAGE_BYTES;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };
  const uint32_t drain_bar = bar0 + 8u * (2 * STAGES + 4);
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(gbase + STAGES * STAGE_BYTES + 8 * (2 * STAGES + 5));
  volatile int *abort = reinterpret_cast<volatile int *>(gbase + STAGES * STAGE_BYTES + 8 * (2 * STAGES + 5) + 8);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), NUM_EPI_WARPS);
    }
    mbar_init(drain_bar, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  MTP_PDL_WAIT();  // barrier init and TMEM allocation above overlap the previous kernel
  MTP_PDL_TRIGGER();
  const uint32_t tmem_base = *tmem_holder;
  const int num_kb = (p.K + BK - 1) / BK;
  // x_proj reduction epilogue over peer memory: the epoch of this reduction (the finishing
  // kernel advances the site's epoch word after this launch, so it cannot change here)
  const uint32_t wire_epoch = (p.wire && p.x.ws > 1) ? *reinterpret_cast<volatile const uint32_t *>(p.x.wepoch) + 1u : 0u;
  const uint32_t tx_bytes = (uint32_t)(A_BYTES + p.bn * BK * 2);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int issued = 0;
      for (int t = blockIdx.x; t < p.num_tiles && !*abort; t += gridDim.x) {
        int mt, nt;
        tile_coords(p, t, mt, nt);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(empty_bar(s), ph ^ 1u, abort, p.timeout_ns)) break;
          mbar_expect_tx(full_bar(s), tx_bytes);
          const uint32_t sa = base + s * STAGE_BYTES;
          tma_load_2d(sa, &tmA, full_bar(s), kb * BK, mt * BM);
          tma_load_2d(sa + A_BYTES, &tmB, full_bar(s), kb * BK, nt * p.bn);
          ++issued;
          if (++s == STAGES) { s = 0; ph ^= 1u; }
        }
      }
      if (*abort) {
        // drain: wait (bounded) until the most recent fills have landed
        int back = issued < STAGES ? issued : STAGES;
        int ss = s;
        uint32_t pp = ph;
        for (int i = 0; i < back; ++i) {
          if (--ss < 0) { ss = STAGES - 1; pp ^= 1u; }
          const unsigned long long t0 = globaltimer_ns();
          while (!mbar_try_wait(full_bar(ss), pp) && globaltimer_ns() - t0 < 100000000ull) {}
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int local = 0;
      bool any = false;
      for (int t = blockIdx.x; t < p.num_tiles && !*abort; t += gridDim.x, ++local) {
        const int a = local & 1;
        const uint32_t use = (uint32_t)(local >> 1);
        if (!mbar_wait(tempty_bar(a), (use & 1u) ^ 1u, abort, p.timeout_ns)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(a * BN_MAX);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(full_bar(s), ph, abort, p.timeout_ns)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = base + s * STAGE_BYTES;
          const uint64_t ad = sw128_desc(sa), bd = sw128_desc(sa + A_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)  // +32 bytes along K per instruction
            umma_bf16(d, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), p.idesc, (kb | k) != 0);
          any = true;
          umma_commit(empty_bar(s));
          if (++s == STAGES) { s = 0; ph ^= 1u; }
        }
        if (!ok) break;
        umma_commit(tfull_bar(a));
      }
      if (*abort && any) {
        umma_commit(drain_bar);
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(drain_bar, 0) && globaltimer_ns() - t0 < 100000000ull) {}
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..13)
    const int q = warp & 3;              // TMEM lane quarter this warp may access
    const int part = (warp - 2) >> 2;    // chunks part, part + EPI_PARTS, ... of the lane quarter
    // TMA-store staging: this warp's 2 KB (two bf16 chunks or one fp32 chunk)
    unsigned char *stage_c = gbase + STAGES * STAGE_BYTES + 256 + (size_t)(warp - 2) * STAGE_C_BYTES;
    const bool dbl = p.c_dtype != MTP_F32;
    int cidx = 0;
    auto emit = [&](int mt, int n0, float (&v)[16], const float (&b)[16]) {
      const int row = mt * BM + q * 32 + lane;
      if (!p.tma_store) {
        epilogue_store(p, row, n0, v, b);
        return;
      }
      epilogue_op(p, v, b);
      const int m0 = mt * BM + q * 32;
      unsigned char *buf = stage_c + (dbl ? (cidx & 1) * 1024 : 0);
      ++cidx;
      // the store that last read this buffer must have finished reading it
      if (lane == 0) {
        if (dbl) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
        else asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
      }
      __syncwarp();
      stage_row(p, buf, lane, v);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> async proxy
      __syncwarp();
      if (lane == 0 && m0 < p.M) tma_store_chunk(&tmC, smem_u32(buf), n0, m0);
    };
    int local = 0;
    if (p.wire) {
      // whole rows per tile: every warp of a lane quarter reads all the row's columns for the
      // row absmax (TMEM reads are cheap; no cross-warp exchange), then writes its own chunks
      const int nch = p.N / 16;
      const unsigned long long half = (wire_epoch & 1u) ? p.x.whalf : 0ull;
      // int8 row block of this lane quarter (32 rows x N <= 192 bytes) in the TMA-store staging area
      unsigned char *wstage = gbase + STAGES * STAGE_BYTES + 256 + (size_t)q * 6144;
      for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++local) {
        const int a = local & 1;
        const uint32_t use = (uint32_t)(local >> 1);
        if (!mbar_wait(tfull_bar(a), use & 1u, abort, p.timeout_ns)) break;
        tc_fence_after();
        int mt, nt;
        tile_coords(p, t, mt, nt);
        const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(a * BN_MAX);
        const int row0 = mt * BM + q * 32, row = row0 + lane;
        if (p.x.ws > 1) {
          // int8 wire to the peers: the part-0 warp of the lane quarter quantises all of its 32
          // rows into shared memory, releases the accumulator, then writes the rows' bytes as one
          // contiguous block per rank (512 bytes per store instruction); the scales of the 32
          // rows are 32 consecutive floats
          if (part == 0) {
            float m = 0.f;
            for (int jc = 0; jc < nch; ++jc) {
              float v[16];
              tmem_ld16(tbase + (uint32_t)(16 * jc), v);
#pragma unroll
              for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(v[i]));
            }
            const float s = row_scale(m);
            for (int jc = 0; jc < nch; ++jc) {
              float v[16];
              tmem_ld16(tbase + (uint32_t)(16 * jc), v);
              uint4 w4;
              w4.x = pack4(quant1(v[0], s), quant1(v[1], s), quant1(v[2], s), quant1(v[3], s));
              w4.y = pack4(quant1(v[4], s), quant1(v[5], s), quant1(v[6], s), quant1(v[7], s));
              w4.z = pack4(quant1(v[8], s), quant1(v[9], s), quant1(v[10], s), quant1(v[11], s));
              w4.w = pack4(quant1(v[12], s), quant1(v[13], s), quant1(v[14], s), quant1(v[15], s));
              *reinterpret_cast<uint4 *>(wstage + (size_t)lane * p.N + 16 * jc) = w4;
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar(a));
            const int nrows = p.M - row0 < 32 ? p.M - row0 : 32;
            if (nrows > 0) {
              const size_t bytes = (size_t)nrows * p.N;
              for (int k = 0; k < p.x.ws; ++k) {
                char *dst = p.x.wslot[(p.x.rank + k) % p.x.ws] + half;  // stagger destinations across ranks
                if (lane < nrows) reinterpret_cast<float *>(dst)[row] = s;
                char *blk = dst + (size_t)4 * p.M + (size_t)row0 * p.N;
                if ((p.M & 3) == 0) {  // 16-byte aligned block
                  for (size_t i = (size_t)lane * 16; i < bytes; i += 512)
                    *reinterpret_cast<uint4 *>(blk + i) = *reinterpret_cast<const uint4 *>(wstage + i);
                } else {
                  for (size_t i = (size_t)lane * 4; i < bytes; i += 128)
                    *reinterpret_cast<uint32_t *>(blk + i) = *reinterpret_cast<const uint32_t *>(wstage + i);
                }
              }
            }
            __syncwarp();  // the staging block is rewritten by the next tile
          } else {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar(a));
          }
          continue;
        }
        // world size 1: the three warps of the lane quarter split the 16-column chunks
        float s = 0.f;
        if (p.x.wmode == MTP_RED_INT8TOK) {
          float m = 0.f;
          for (int jc = 0; jc < nch; ++jc) {
            float v[16];
            tmem_ld16(tbase + (uint32_t)(16 * jc), v);
#pragma unroll
            for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(v[i]));
          }
          s = row_scale(m);
        }
        for (int jc = part; jc < nch; jc += EPI_PARTS) {
          float v[16];
          tmem_ld16(tbase + (uint32_t)(16 * jc), v);
          if (row < p.M) wire_chunk_local(p, row, 16 * jc, v, s);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty_bar(a));
      }
    }
    for (int t = blockIdx.x; t < (p.wire ? 0 : p.num_tiles); t += gridDim.x, ++local) {
      const int a = local & 1;
      const uint32_t use = (uint32_t)(local >> 1);
      if (!mbar_wait(tfull_bar(a), use & 1u, abort, p.timeout_ns)) break;
      tc_fence_after();
      int mt, nt;
      tile_coords(p, t, mt, nt);
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(a * BN_MAX);
      // this warp's 16-column chunks are j, j + 16 EPI_PARTS, ...: two per TMEM wait
      constexpr int CS = 16 * EPI_PARTS;
      for (int j = part * 16; j < p.bn; j += 2 * CS) {
        const int n0 = nt * p.bn + j;
        const bool two = j + CS < p.bn;  // warp-uniform
        float b[16], b2[16];
        if (p.epi != MTP_EPI_STORE) {  // issued before the TMEM read
          if (n0 < p.N) load_bias16(p, n0, b);
          if (two && n0 + CS < p.N) load_bias16(p, n0 + CS, b2);
        }
        float v[16], v2[16];
        if (two) {
          tmem_ld16x2(tbase + (uint32_t)j, tbase + (uint32_t)(j + CS), v, v2);
        } else {
          tmem_ld16(tbase + (uint32_t)j, v);
        }
        if (n0 < p.N) emit(mt, n0, v, b);
        if (two && n0 + CS < p.N) emit(mt, n0 + CS, v2, b2);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(a));
    }
    // every TMA store of this warp has completed before the CTA exits
    if (p.tma_store && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0 && *abort) atomicExch(p.err, MTP_ERR_TIMEOUT);
  // x_proj reduction over peer memory: every epilogue store of this CTA is ordered before
  // the flags by the barrier above, then one system fence and release store per rank
  if (p.wire && p.x.ws > 1 && threadIdx.x < (unsigned)p.x.ws && !*abort) {
    __threadfence_system();
    st_release_sys(p.x.wflag[threadIdx.x] + blockIdx.x, wire_epoch);
  }
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
}

// ------------------------------------------------------------------ host side
static int *device_err_word() {
  static int *w = nullptr;  // one word per process (single device per process)
  if (!w) {
    if (cudaMalloc(&w, sizeof(int)) != cudaSuccess) return nullptr;
    cudaMemset(w, 0, sizeof(int));
  }
  return w;
}

}  // namespace tc

// True when the operands satisfy the TMA rules of this kernel.
bool gemm_tc_eligible(const void *A, const void *B, int M, int N, int K, int lda, int ldb) {
  return M > 0 && N > 0 && K >= 8 && aligned16(A) && aligned16(B) && lda % 8 == 0 && ldb % 8 == 0 && lda >= K &&
         ldb >= K;
}

int gemm_tc(const void *A, const void *B, void *C, int M, int N, int K, int lda, int ldb, int ldc, int c_dtype,
            int epi, const void *bias, int bias_dtype, cudaStream_t stream) {
  using namespace tc;
  MTP_REQUIRE(gemm_tc_eligible(A, B, M, N, K, lda, ldb),
              "tcgen05 GEMM needs 16-byte aligned A/B, K >= 8 and lda, ldb multiples of 8");
  MTP_REQUIRE(c_dtype == MTP_F32 || c_dtype == MTP_BF16, "C must be F32 or BF16");
  MTP_REQUIRE(epi == MTP_EPI_STORE || ((epi == MTP_EPI_BIAS_SOFTPLUS || epi == MTP_EPI_BIAS) && bias), "bad epilogue");
  Params p{};
  p.C = C;
  p.bias = bias;
  p.bias_dtype = bias_dtype;
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldc = ldc;
  p.c_dtype = c_dtype;
  p.epi = epi;
  p.bn = N <= BN_MAX ? ((N + 15) / 16) * 16 : BN_MAX;
  p.tiles_m = ceil_div(M, BM);
  // few M tiles (small batches): narrower N tiles so the grid still covers the SMs
  const int sms_avail = num_sms();
  while (p.bn > 32 && (long)p.tiles_m * ceil_div(N, p.bn) < sms_avail) p.bn = ((p.bn / 2 + 15) / 16) * 16;
  p.tiles_n = ceil_div(N, p.bn);
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.group_m = 32;
  p.idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(p.bn >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
  const size_t cb = c_dtype == MTP_F32 ? 4 : 2;
  p.vec_ok = aligned16(C) && ((size_t)ldc * cb) % 16 == 0;
  p.timeout_ns = 2000000000ull;
  p.err = device_err_word();
  if (!p.err) return fail(MTP_ERR_CUDA, "could not allocate the GEMM status word");
  CUtensorMap ta, tb, tcm;
  int rc = make_tmap(&ta, A, M, K, lda, BM);
  if (rc) return rc;
  rc = make_tmap(&tb, B, N, K, ldb, p.bn);
  if (rc) return rc;
  // epilogue through shared memory and TMA stores (MTP_GEMM_TMA_STORE=0: direct stores)
  static const bool tma_store_on = [] {
    const char *e = getenv("MTP_GEMM_TMA_STORE");
    return !(e && e[0] == '0');
  }();
  p.tma_store = tma_store_on && p.vec_ok && N >= 16 && M >= 32;
  memset(&tcm, 0, sizeof(tcm));
  if (p.tma_store) {
    rc = make_tmap_c(&tcm, C, M, N, ldc, c_dtype);
    if (rc) return rc;
  }
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES_TMA_STORE);
    attr = true;
  }
  const int grid = p.num_tiles < num_sms() ? p.num_tiles : num_sms();
  launch_pdl(gemm_tc_kernel, dim3(grid), dim3(NUM_THREADS), p.tma_store ? SMEM_BYTES_TMA_STORE : SMEM_BYTES, stream,
             ta, tb, tcm, p);
  return check_launch("gemm_tc");
}

// The x_proj GEMM with the reduction epilogue (wire_chunk_local, the int8 row blocks): C is not written.  Returns
// the grid size through *grid_out (the finishing kernel waits for that many CTAs per rank).
int gemm_tc_xproj_wire(const void *A, const void *B, int M, int N, int K, int lda, int ldb, const XprojWire &w,
                       int *grid_out, cudaStream_t stream) {
  using namespace tc;
  MTP_REQUIRE(gemm_tc_eligible(A, B, M, N, K, lda, ldb),
              "tcgen05 GEMM needs 16-byte aligned A/B, K >= 8 and lda, ldb multiples of 8");
  MTP_REQUIRE(N % 16 == 0 && N <= 192 && w.R % 16 == 0 && w.R > 0 && w.R < N, "x_proj epilogue: bad widths");
  MTP_REQUIRE(w.ws <= 1 || w.wmode == MTP_RED_INT8TOK, "x_proj epilogue over peer memory: int8 wire only");
  static_assert(NUM_EPI_WARPS * STAGE_C_BYTES >= 4 * 6144, "staging area holds four 32 x 192-byte row blocks");
  Params p{};
  p.x = w;
  p.wire = 1;
  p.C = nullptr;
  p.bias = nullptr;
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldc = N;
  p.c_dtype = MTP_F32;
  p.epi = MTP_EPI_STORE;
  p.bn = N;  // one N tile: whole rows
  p.tiles_m = ceil_div(M, BM);
  p.tiles_n = 1;
  p.num_tiles = p.tiles_m;
  p.group_m = 32;
  p.idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(p.bn >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
  p.vec_ok = 0;
  p.tma_store = 0;
  p.timeout_ns = 2000000000ull;
  p.err = device_err_word();
  if (!p.err) return fail(MTP_ERR_CUDA, "could not allocate the GEMM status word");
  CUtensorMap ta, tb, tcm;
  int rc = make_tmap(&ta, A, M, K, lda, BM);
  if (rc) return rc;
  rc = make_tmap(&tb, B, N, K, ldb, p.bn);
  if (rc) return rc;
  memset(&tcm, 0, sizeof(tcm));
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES_TMA_STORE);
    attr = true;
  }
  const int grid = p.num_tiles < num_sms() ? p.num_tiles : num_sms();
  *grid_out = grid;
  // the peer path stages int8 row blocks in the TMA-store staging area (4 x 6 KB)
  launch_pdl(gemm_tc_kernel, dim3(grid), dim3(NUM_THREADS), w.ws > 1 ? SMEM_BYTES_TMA_STORE : SMEM_BYTES, stream, ta,
             tb, tcm, p);
  return check_launch("gemm_tc_xproj");
}

int gemm_tc_status(int *status) {
  int *w = tc::device_err_word();
  if (!w) return fail(MTP_ERR_CUDA, "no status word");
  if (cudaMemcpy(status, w, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return fail(MTP_ERR_CUDA, "read status");
  return MTP_OK;
}

}  // namespace mtp
