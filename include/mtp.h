/*
 * mtp.h -- C ABI of libmtp.so, the B200 (sm_100a) kernels behind the
 * channel-sharded tensor-parallel Mamba-1 forward pass.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), returns an int status (0 = ok, see MTP_ERR_*) and launches
 * only on the given stream.  Device memory is allocated by the create / bind
 * calls (mtp_comm_create, mtp_decode_plan_create, mtp_decode_bind_cache) and,
 * on first use, for four internal buffers kept until exit: a status word of
 * the tensor-core GEMM, one of the fused dt_proj scan, the row scratch of
 * the reductions that do not hold a row in registers (rows wider than 3072
 * values or not a multiple of 4, a grid capped by mtp_comm_set_max_ctas, or a
 * per-tensor-scale mode), and the state scratch of the sequence-chunked scan;
 * the last two grow to the largest size used.  A call that is to be recorded in a
 * CUDA graph therefore needs one call of the same kind before the capture (the
 * package's GraphedStepper runs warm-up steps first).  No torch types appear
 * here; the Python package binds this header with ctypes.
 *
 * Devices: the library serves one device per process (one rank per process), except
 * the allocation-free reduction scratch, the reductions' row scratch and the chunked
 * scan's state scratch, which are kept per device; the status words of the GEMM and of the fused scan are per process.
 *
 * Layout conventions: matrices are row-major; a "token row" is one position
 * of one sequence, tokens ordered (batch, position).  Element type codes are
 * MTP_F32 / MTP_BF16 / MTP_F16.
 *
 * Each function names the reference (Mamba-TP Lite, pure PyTorch) code it
 * replaces, as path:line within that project.
 */
#ifndef MTP_H_
#define MTP_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  MTP_OK = 0,
  MTP_ERR_ARG = 1,         /* bad size, pointer, stride or alignment */
  MTP_ERR_CUDA = 2,        /* a CUDA runtime call or launch failed */
  MTP_ERR_TIMEOUT = 3,     /* a bounded device wait expired (peer never arrived) */
  MTP_ERR_UNSUPPORTED = 4  /* combination not built (dtype, size class) */
};

enum { MTP_F32 = 0, MTP_BF16 = 1, MTP_F16 = 2 };

/* Reduction (collective) wire modes: the reference's ALLREDUCE_FNS names
 * (mamba_lite/tp_utils.py:152-160): "fp32", "fp16", "int8" (== "int8_gather_tok"), and
 * the per-tensor-scale variants "int8_gather" (:134-142), "int8_sum" (:78-100) and
 * "int8_legacy" (:45-75). */
enum {
  MTP_RED_FP32 = 0,
  MTP_RED_FP16 = 1,
  MTP_RED_INT8TOK = 2,
  MTP_RED_INT8TENSOR = 3, /* one scale per rank's tensor, int8 gathered, rank-ordered dequant-sum */
  MTP_RED_INT8SUM = 4,    /* scale shared by all ranks (MAX), values in +-(127 / ws), integer sum */
  MTP_RED_INT8LEGACY = 5  /* scale shared by all ranks (MAX), values in +-127, integer sum */
};

/* GEMM epilogues. */
enum {
  MTP_EPI_STORE = 0,         /* C = acc                                   */
  MTP_EPI_BIAS_SOFTPLUS = 1, /* C = softplus(acc + bias[n]) (torch threshold 20) */
  MTP_EPI_BIAS = 2           /* C = acc + bias[n]                          */
};

/* GEMM algorithm selector (mtp_gemm_ex).  AUTO picks TCGEN05 for bf16 with
 * M > 16 and TMA-compatible strides, GEMV for M <= 64 otherwise, SIMT for the rest. */
enum { MTP_GEMM_AUTO = 0, MTP_GEMM_TCGEN05 = 1, MTP_GEMM_SIMT = 2, MTP_GEMM_GEMV = 3 };

const char *mtp_version(void);
/* Text of the last host-side error of the calling thread ("" if none). */
const char *mtp_last_error(void);
/* Number of kernel launches issued by this library since load (all threads). */
uint64_t mtp_launch_count(void);

/* ------------------------------------------------------------------ GEMM
 * C[M,N] = A[M,K] . B[N,K]^T, fp32 accumulation, optional epilogue.
 * A: activations (a_dtype), B: weights (same dtype as A), C: c_dtype.
 * Replaces nn.Linear / F.linear on the hot path:
 *   in_proj  mamba_lite/tp_model.py:91, :142   (model.py:197, :261)
 *   x_proj   tp_model.py:106, :159             (model.py:214, :279)
 *   dt_proj  tp_model.py:110-111, :162-163 with MTP_EPI_BIAS_SOFTPLUS
 *   out_proj tp_model.py:131, :175             (model.py:239, :293)
 *   lm_head  tp_model.py:302-303               (model.py:325-326)
 */
int mtp_gemm(const void *A, const void *B, void *C, int M, int N, int K, int lda, int ldb, int ldc,
             int ab_dtype, int c_dtype, int epilogue, const void *bias, int bias_dtype, void *stream);
int mtp_gemm_ex(const void *A, const void *B, void *C, int M, int N, int K, int lda, int ldb, int ldc,
                int ab_dtype, int c_dtype, int epilogue, const void *bias, int bias_dtype, int algo,
                void *stream);

/* ------------------------------------------------------------------ SSM
 * Causal depthwise conv1d + SiLU over the x half of in_proj's output.
 * xz: [B*L, ld_xz] (x in columns [0,Es)); conv_w [Es,K]; conv_b [Es] or NULL;
 * hist: [B,Es,K-1] prior conv history or NULL (zeros); xc: [B*L, ld_xc].
 * Pure (writes only xc); the fused scan / step kernels own the cache update.
 * Replaces tp_model.py:93-100 (model.py:199-209) and the conv part of
 * tp_model.py:145-157.  dtype: activation / parameter type (F32 or BF16). */
int mtp_conv1d_silu(const void *xz, int ld_xz, const void *conv_w, const void *conv_b,
                    const void *hist, void *xc, int ld_xc, int B, int L, int Es, int K, int dtype,
                    void *stream);

/* Fused prefill: causal conv1d + SiLU + selective scan + D skip + SiLU(z) gate.
 * xz: [B*L, ld_xz] (x | z); dt: [B*L, ld_dt] in dt_dtype (F32, or the model dtype
 * as the reference's bf16 dt_proj output), softplus already applied;
 * bc: [B*L, ld_bc] fp32 with B in columns [0,N) and C in [N,2N);
 * A_log [Es,N], D [Es], conv_w [Es,K], conv_b [Es] in dtype;
 * conv_init [B,Es,K-1] (dtype) / ssm_init [B,Es,N] (fp32) or NULL for zeros;
 * y: [B*L, ld_y] (dtype); conv_final [B,Es,K-1] (dtype), ssm_final [B,Es,N] (fp32).
 * conv_final may alias conv_init and ssm_final may alias ssm_init (in-place
 * chunked prefill).  Replaces tp_model.py:93-103 and :113-129
 * (model.py:199-241), the Python loop over t at tp_model.py:124-126. */
int mtp_scan_prefill(const void *xz, int ld_xz, const void *dt, int ld_dt, int dt_dtype, const float *bc, int ld_bc,
                     const void *A_log, const void *Dp, const void *conv_w, const void *conv_b,
                     const void *conv_init, const float *ssm_init, void *y, int ld_y, void *conv_final,
                     float *ssm_final, int B, int L, int Es, int N, int K, int dtype, void *stream);

/* The selective scan of mtp_scan_prefill fed with the conv output instead of raw x:
 * xc [B*L, ld_xc] = SiLU(conv1d(x)) as written by mtp_conv1d_silu (the x_proj input,
 * computed once per layer); z is read from columns [Es, 2Es) of xz and the raw x
 * columns [0, Es) of xz only for the final conv history.  Other arguments as
 * mtp_scan_prefill (conv weights are not needed).  With few recurrences (B x Es <= 8192)
 * over long sequences (L >= 2048) the sequence is cut into up to 16 chunks: a state pass
 * gives each chunk's end state from zero and its sum of dt, and each chunk's output pass
 * starts from the state carried through the earlier chunks (MTP_SCAN_CHUNKS=n forces n
 * chunks; the results agree with the unchunked scan to rounding).  State pairs are updated with
 * packed fp32 arithmetic; optionally (MTP_SCAN_POLY pairs per thread, 0 by default) part
 * of the state exponentials is evaluated on the FP32 pipe (the polynomial of mtp_exp2_fma).  Replaces tp_model.py:101-103 and :113-129
 * (model.py:210-241), the Python loop over t at tp_model.py:124-126. */
int mtp_scan_prefill_xc(const void *xc, int ld_xc, const void *xz, int ld_xz, const void *dt, int ld_dt,
                        int dt_dtype, const float *bc, int ld_bc, const void *A_log, const void *Dp,
                        const void *conv_init, const float *ssm_init, void *y, int ld_y, void *conv_final,
                        float *ssm_final, int B, int L, int Es, int N, int K, int dtype, void *stream);
/* out[i] = 2^x[i] for x[i] <= 0 by the FP32-pipe polynomial that mtp_scan_prefill_xc
 * uses for part of exp(dt * A) (x < -125 gives 2^-125).  Test entry: the reference
 * computes these factors with torch.exp (tp_model.py:114). */
int mtp_exp2_fma(const float *x, float *out, int n, void *stream);

/* The fused prefill above with dt_proj folded in (bf16 models): dt = softplus(
 * dt_low . W_dt^T + b_dt) is computed inside the kernel on the tensor cores
 * (tcgen05.mma, TMEM accumulators) instead of being read from memory.
 * dt_low [B*L, ld_dl] bf16 (R values per row), W_dt [Es, R] bf16, b_dt [Es] bf16;
 * other arguments as mtp_scan_prefill (all bf16 except bc / ssm states).  Needs
 * d_state 16, Es % 128 == 0, R % 8 == 0 and R <= 256.  Replaces
 * tp_model.py:110-129 (model.py:216-238).  A bounded internal wait that expires
 * sets the status read by mtp_scan_status. */
int mtp_scan_prefill_fused(const void *xz, int ld_xz, const void *dt_low, int ld_dl, const void *W_dt,
                           const void *b_dt, const float *bc, int ld_bc, const void *A_log, const void *Dp,
                           const void *conv_w, const void *conv_b, const void *conv_init, const float *ssm_init,
                           void *y, int ld_y, void *conv_final, float *ssm_final, int B, int L, int Es, int N, int R,
                           int K, void *stream);
/* Device status of the fused scan (0, or MTP_ERR_TIMEOUT after an expired wait). */
int mtp_scan_status(int *status);

/* Single-token recurrent step, in place: conv history shift, SiLU, dt_proj
 * (dt_low . W_dt^T + b) and softplus, state update, y = C.h + D.x, SiLU(z) gate.
 * xz [B, ld_xz]; dt_low [B, ld_dl] (R values, dtype) ; W_dt [Es,R], b_dt [Es];
 * bc [B, ld_bc] fp32 (B | C); conv_state [B,Es,K-1] (dtype) and ssm_state
 * [B,Es,N] (fp32) are read and overwritten; y [B, ld_y].
 * Replaces tp_model.py:145-173 (model.py:264-292); in-place copy_ at
 * tp_model.py:154 and :170. */
int mtp_step(const void *xz, int ld_xz, const void *dt_low, int ld_dl, const void *W_dt, const void *b_dt,
             const float *bc, int ld_bc, const void *A_log, const void *Dp, const void *conv_w,
             const void *conv_b, void *conv_state, float *ssm_state, void *y, int ld_y, int B, int Es,
             int N, int R, int K, int dtype, void *stream);

/* ------------------------------------------------------------------ misc
 * Embedding gather (tp_model.py:308, :318): out[t,:] = table[ids[t],:] (fp32 out).
 * ids are int64. */
int mtp_embedding(const int64_t *ids, int T, const void *table, int D, int dtype, float *out, void *stream);
/* RMSNorm (model.py:130-135): out = w * (x * rsqrt(mean(x^2) + eps)), x fp32
 * [T, D], out in out_dtype. */
int mtp_rmsnorm(const float *x, int T, int D, const void *w, int w_dtype, float eps, void *out,
                int out_dtype, void *stream);
/* Row-wise argmax of logits [T, V] (dtype) -> int64 (greedy decode, model.py:359/:363). */
int mtp_argmax_rows(const void *logits, int T, int V, int ld, int dtype, int64_t *out, void *stream);

/* ------------------------------------------------------------------ quantiser
 * Per-row int8 quantiser of the "int8" collective (tp_utils.py:108-113):
 * scale = max(amax|row|, 1e-8) / 127 (IEEE fp32 divide), q = clamp(rint(x / scale), +-127).
 * Same device function as the one inside mtp_reduce_*; exported so tests can
 * compare payload bytes with the reference bit for bit. */
int mtp_quantize_rows_int8(const float *in, int rows, int cols, int ld, float *scales, int8_t *q,
                           void *stream);
/* Rank-ordered dequant-sum of packed payloads [ws][rows*4 scale bytes | rows*cols q]
 * (tp_utils.py:127-130), product rounded before the add. */
int mtp_dequant_sum(const uint8_t *payloads, int ws, int rows, int cols, float *out, void *stream);

/* ------------------------------------------------------------------ collectives
 * A comm context owns, per reduction site kind (0 = x_proj, 1 = out_proj),
 * receive slots for every rank, a gather buffer, flag words and epoch
 * counters in one device allocation that peers map through CUDA IPC.
 * Bootstrap: mtp_comm_create on every rank, exchange the 64-byte handles
 * (mtp_comm_ipc_handle) out of band, mtp_comm_open_peers, then a host
 * barrier before the first reduction.  world_size 1 needs no context (pass
 * NULL to the reduce calls).  Replaces the NCCL/gloo calls of
 * tp_utils.py:27, :41, :120/:124. */
typedef struct mtp_comm mtp_comm;
int mtp_comm_create(int rank, int world_size, int max_rows, int cols_x, int cols_out, double timeout_s,
                    mtp_comm **out);
int mtp_comm_ipc_handle(mtp_comm *c, void *handle64);
int mtp_comm_open_peers(mtp_comm *c, const void *handles /* world_size x 64 bytes */);
int mtp_comm_destroy(mtp_comm *c);
/* Device status word of the context: 0 ok, else MTP_ERR_TIMEOUT (host reads it
 * after a synchronize; a timed-out reduction leaves its outputs undefined). */
int mtp_comm_status(mtp_comm *c, int *status);
int mtp_comm_reset_status(mtp_comm *c);
/* Recovery after MTP_ERR_TIMEOUT: zeroes the context's flags, epochs, exit counters and
 * status word.  A timed-out reduction or decode step leaves flags and epochs that no longer
 * agree across ranks, so with no kernel in flight on any rank, every rank calls this (and
 * mtp_decode_reset on its decode plan), then the ranks meet at a host barrier before the
 * next reduction or step. */
int mtp_comm_reset_state(mtp_comm *c);
/* Launch shape of the context's reductions: max_ctas > 0 caps a reduction's grid at
 * max_ctas CTAs and selects the low-register kernel variant, so a reduction can run
 * on the SMs beside a GEMM or scan of another stream (compute/communication overlap
 * across micro-batches); 0 restores the default (one CTA per SM, register rows).
 * Results are bit-identical either way. */
int mtp_comm_set_max_ctas(mtp_comm *c, int max_ctas);

/* Sequence-parallel out_proj epilogue on this context (default on): at world size > 1 each
 * row's owner rank (row % ws) applies the bias, residual and next RMSNorm and the normed rows
 * are gathered, so a rank's residual stays current only on its own rows.  A model whose
 * out_proj sites mix modes with and without that form (the per-tensor-scale modes have no
 * such form) turns it off for its forward passes, so every reduction updates every row. */
int mtp_comm_set_sequence_parallel(mtp_comm *c, int on);

/* Bytes this rank sends to its peers over NVLink for one reduction of [rows, cols] in
 * `mode` whose results are rounded to rdt (MTP_F32 / MTP_BF16), with the protocol the
 * reduce calls choose (0 without a context or at world size 1).  For bandwidth reports;
 * the reference counts payload bytes per call at tp_utils.py:24-26, :38-40, :114-116. */
int mtp_comm_sent_bytes(mtp_comm *c, int mode, int rows, int cols, int rdt, double *bytes);

/* Phase trace of the pipelined reductions on this context (diagnostics; off by default).
 * records > 0 allocates a ring of that many launch records of 131 uint64 each: [0] grid
 * size, [1] rounds, [2] bit 0: the two-shot protocol, bits 8+: the site, then from [3] (CTA 0) and [67] (the
 * last CTA) the %globaltimer ns at start and after each push / wait / reduce / signal
 * step of each round; 0 frees it.  Not allowed while a reduction is in flight. */
int mtp_comm_set_trace(mtp_comm *c, int records);
int mtp_comm_read_trace(mtp_comm *c, uint64_t *out, int capacity, int *n_records);

/* AllReduce #1 epilogue (tp_model.py:106-108, :159-161): sum the fp32
 * partial [rows, R+2N] over ranks in `mode`, round the sums to dt_dtype (the
 * reference's reduction returns the model dtype, tp_utils.py:42, :131), then
 * split: dt_low [rows, R] (dt_dtype, input of dt_proj) and bc [rows, 2N] fp32
 * (scan input). */
int mtp_reduce_xproj(mtp_comm *c, int mode, const float *partial, int rows, int R, int N2,
                     void *dt_low, int dt_dtype, float *bc, void *stream);
/* AllReduce #2 epilogue (tp_model.py:131-134 then the block residual
 * tp_model.py:254-257 and the next RMSNorm): out = sum over ranks of the fp32
 * partial [rows, D] rounded to out_dtype (the reduction's return dtype) (+ bias),
 * resid += out (fp32, in place), and normed = RMSNorm(resid) * norm_w in
 * out_dtype (skipped when normed is NULL). */
int mtp_reduce_outproj(mtp_comm *c, int mode, const float *partial, int rows, int D, const void *bias,
                       float *resid, const void *norm_w, float eps, void *normed, int out_dtype,
                       void *stream);
/* x_proj GEMM fused with AllReduce #1 (tp_model.py:106-108: x_dbl = x_proj(x), reduced
 * across ranks, split into dt | B | C): partial = xc[rows, K] . w[N, K]^T (bf16 operands,
 * fp32 accumulate) is never written; the GEMM's epilogue quantises / casts each row to the
 * wire format of `mode` and, at world size 1, applies the wire round trip and writes
 * dt_low [rows, R] (dt_dtype, also the rounding dtype of the reduced values) and bc
 * [rows, N-R] fp32 directly; at world size > 1 it writes the wire rows into every rank's
 * receive slot of the x_proj site and flags them, and a second kernel reduces every row
 * over the ranks in rank order and splits it.  xc and w are ab_dtype (the fused form
 * needs MTP_BF16).  Bit-identical to mtp_gemm into `partial`
 * followed by mtp_reduce_xproj, which is what runs when the shape does not fit the fused
 * form (N % 16, N <= 192, R % 16, 16-byte aligned operands and outputs; at world size > 1
 * the int8 wire only, rows within the context's slots, no grid cap; by default only at world
 * sizes 1 and 2, whose one-shot push is not larger than the two-shot protocol's traffic, and
 * with at least 64 x (SM count) rows;
 * MTP_XPROJ_FUSED=1 / 0 forces the fused form / the kernel pair): `partial` [rows, N] fp32 is
 * only used then and may be NULL for shapes that fit. */
int mtp_xproj_fused(mtp_comm *c, int mode, const void *xc, int ld_xc, const void *w, int ld_w, int ab_dtype, int rows,
                    int N, int K, int R, float *partial, void *dt_low, int dt_dtype, float *bc, void *stream);
/* Plain reduction (the isolated site of the collective microbenchmark):
 * out[rows, cols] (fp32) = reduce(in) over ranks; site selects the buffers. */
int mtp_allreduce(mtp_comm *c, int site, int mode, const float *in, float *out, int rows, int cols,
                  void *stream);

/* Allocation-free form of the world-size-1 case of mtp_allreduce (no comm
 * context): the wire-format round trip of `mode` (fp32 copy, fp16 cast,
 * int8-per-row quantise/dequantise) of in[rows, cols] into out, bit-identical
 * to mtp_allreduce(NULL, ...).  No counterpart in the reference: it exists for
 * callers that cannot call cudaMalloc at all -- for instance code running
 * inside a host-side memory budget or a runtime that owns every device
 * allocation -- whereas mtp_allreduce may allocate its row scratch on first use.
 * Its scratch is a fixed 4 MiB file-scope device array (1 Mi floats) that every
 * GPU loading the library holds until process exit, so rows wider than 131072
 * values are rejected with MTP_ERR_ARG.  The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress); make that first call before
 * any stream capture.  All calls share the array and nothing in it needs to
 * start at zero (each row is written before it is read), but calls that overlap
 * on the GPU (different streams, different host threads) race on it. */
int mtp_allreduce_noalloc(int mode, const float *in, float *out, int rows, int cols, void *stream);

/* ---------------------------------------------------------------- vocabulary-parallel lm_head
 * The reference replicates the tied lm_head on every rank (TPMambaLM.lm_head,
 * tp_model.py:302-303: logits = x @ embedding.weight^T, every rank reading all V rows).
 * Vocabulary-parallel form: rank k computes only logits columns [col0, col0 + cols)
 * (mtp_vocab_shard: ceil(V / ws) rounded up to a multiple of 8, the last rank the
 * remainder) and the ranks exchange their columns over the context's peer memory, so
 * every rank returns the full [rows, V] logits, bit-identical to the replicated GEMM
 * (same kernel and summation order per element).  Used for few rows (decode steps):
 * each rank then reads V / ws embedding rows instead of V.  normed [rows, K], emb
 * [V, K] (the tied embedding), out [rows, V], all of `dtype` (MTP_F32 / MTP_BF16).
 * rows x shard x element size must fit one receive slot of the out_proj site
 * (max_rows x (4 cols_out + 16) bytes).  c NULL or world size 1: the plain GEMM.
 * Collective: every rank calls it with the same rows, V and dtype. */
int mtp_vocab_shard(int V, int world_size, int rank, int *col0, int *cols);
int mtp_lm_head_vocab_parallel(mtp_comm *c, const void *normed, int rows, int K, int ld_normed, const void *emb, int V,
                               int ld_emb, int dtype, void *out, int ld_out, void *stream);

/* ---------------------------------------------------------------- persistent decode
 * One cooperative launch per decode step runs every layer of the model for a batch
 * of single tokens: embedding gather (tp_model.py:318), per layer the block's
 * RMSNorm and residual (tp_model.py:259-262) around the TPMambaMixer.step sequence
 * (tp_model.py:137-179) with both AllReduces in the layer's wire format over the
 * comm context (tp_utils.py:23-42, :103-131), and finally norm_f (tp_model.py:321);
 * the caller runs the lm_head GEMM on `normed`.  It replaces the loop over layers of
 * TPMambaLM.step / MambaLM.step (tp_model.py:317-322, model.py:343-353): one launch
 * instead of seven per layer.  bf16 models, d_state 16, d_conv 4, batch <= 32. */
typedef struct mtp_decode_plan mtp_decode_plan;
typedef struct mtp_decode_cache mtp_decode_cache;

typedef struct {
  const void *norm_w;          /* [D]        RMSNorm weight in front of the mixer        */
  const void *in_w, *in_b;     /* [2Es, D]   in_proj (this rank's x rows then z rows); bias or NULL */
  const void *conv_w, *conv_b; /* [Es, K], [Es] or NULL                                   */
  const void *x_w;             /* [R+2N, Es] x_proj (this rank's input columns)            */
  const void *dt_w, *dt_b;     /* [Es, R], [Es]                                            */
  const void *A_log, *Dp;      /* [Es, N], [Es]                                            */
  const void *out_w, *out_b;   /* [D, Es] out_proj (this rank's input columns); bias or NULL */
  int mode_x, mode_out;        /* MTP_RED_* wire format of AllReduce #1 / #2               */
} mtp_decode_layer;

/* Validates shapes, copies the layer table to the device and allocates the step's
 * scratch for up to max_batch tokens.  comm NULL (or world size 1) runs each
 * AllReduce as its wire format's round trip. */
int mtp_decode_plan_create(const mtp_decode_layer *layers, int n_layer, const void *norm_f, const void *embedding,
                           int d_model, int d_inner, int d_state, int dt_rank, int d_conv, float eps, int max_batch,
                           int dtype, mtp_comm *comm, mtp_decode_plan **out);
/* Binds per-layer cache tensors: conv_state[l] [batch][Es][K-1] (model dtype) and
 * ssm_state[l] [batch][Es][N] fp32, both updated in place by each step. */
int mtp_decode_bind_cache(mtp_decode_plan *plan, void *const *conv_state, float *const *ssm_state, int batch,
                          mtp_decode_cache **out);
/* ids: device int64 [batch]; normed: device [batch][D] model dtype, receives
 * norm_f(residual stream) of the step. */
int mtp_decode_step(mtp_decode_plan *plan, mtp_decode_cache *cache, const int64_t *ids, void *normed, void *stream);
/* MTP_OK, or MTP_ERR_TIMEOUT after a barrier or peer wait gave up (synchronous read). */
int mtp_decode_status(mtp_decode_plan *plan, int *status);
/* Clears the barrier, abort, status and per-row flag words after a timeout (synchronous).
 * The comm context needs mtp_comm_reset_state on every rank as well before the next step. */
int mtp_decode_reset(mtp_decode_plan *plan);
/* Phase timing of later steps (off by default): with tracing on, each step stores
 * nb = 2 + 5 n_layer %globaltimer stamps of CTA 0: out[0] = start, out[1] = end of
 * the embedding phase, then the end of each of the five phases of every layer
 * (in_proj+conv, x_proj, AllReduce #1 + step, out_proj, AllReduce #2 + norm). */
int mtp_decode_set_trace(mtp_decode_plan *plan, int on);
int mtp_decode_read_trace(mtp_decode_plan *plan, uint64_t *out, int capacity, int *n_out);
void mtp_decode_cache_destroy(mtp_decode_cache *cache);
void mtp_decode_plan_destroy(mtp_decode_plan *plan);

#ifdef __cplusplus
}
#endif
#endif /* MTP_H_ */
