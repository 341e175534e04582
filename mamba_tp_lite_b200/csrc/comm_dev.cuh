// Layout of a comm context (one cudaMalloc per rank, mapped by its peers over CUDA IPC),
// shared by the reduction kernels (comm.cu) and the persistent decode kernel (decode.cu).
//   flags   u32 [site 2][phase 4][src MAX_WS][G_MAX]   phases 0-1: value = epoch of the last push (scratch
//                                                      kernel, decode); 2-3: epoch * 256 + round (pipelined kernel)
//   epoch   u32 [site 2]                              last completed epoch per site
//   done    u32 [site 2]                              CTA exit counter of a reduction launch
//   status  int                                        MTP_OK or MTP_ERR_TIMEOUT
//   recv[s] 2 halves (epoch parity) x ws slots of slot_bytes[s]: the wire rows pushed by each rank
//   gath[s] max_rows x cols[s] fp32: reduced rows of the two-shot protocol
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace mtp {

constexpr int MAX_WS = 8;
constexpr int G_MAX = 512;  // CTAs of one reduction launch (flag slots per source rank)
constexpr int NPHASE = 4;   // flag phases per site

// Phase trace of the pipelined reductions (off unless mtp_comm_set_trace allocated it):
// per launch one record of TRACE_WORDS u64 written by thread 0 of CTA 0 and of the last
// CTA: [0] grid, [1] rounds, [2] protocol (bit 0) and site (bits 8+); then per CTA (CTA 0 at 3, the last at 3 + 64)
// the %globaltimer at start and after each event of each round.
constexpr int TRACE_WORDS = 131;

struct CommDev {
  char *peer[MAX_WS];  // base of each rank's allocation (peer[rank] = own)
  size_t off_flags, off_epoch, off_done, off_status, off_recv[2], off_gath[2], slot_bytes[2];
  int rank, ws;
  unsigned long long timeout_ns;
  unsigned long long *trace;  // [trace_cap][TRACE_WORDS] or NULL
  unsigned int *trace_count;  // launches recorded (the record index is count % trace_cap)
  int trace_cap;
};

__device__ __forceinline__ uint32_t *flag_ptr(char *base, const CommDev &d, int site, int phase, int src, int j) {
  return reinterpret_cast<uint32_t *>(base + d.off_flags) + (((size_t)(site * NPHASE + phase) * MAX_WS + src) * G_MAX + j);
}

}  // namespace mtp

struct mtp_comm {
  mtp::CommDev d;
  char *base = nullptr;
  size_t total = 0;
  int max_rows = 0, cols[2] = {0, 0};
  int max_ctas = 0;  // > 0: cap on a reduction's grid, low-register kernel (runs beside compute kernels)
  bool sp_allowed = true;  // sequence-parallel out_proj epilogue (mtp_comm_set_sequence_parallel)
  bool opened = false;
  cudaIpcMemHandle_t handle;
};
