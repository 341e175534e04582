// Host error plumbing, embedding gather, RMSNorm, row argmax.
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include "common.cuh"

namespace mtp {

static thread_local std::string t_last_error;
std::atomic<uint64_t> g_launches{0};

void set_error(const std::string &msg) { t_last_error = msg; }

int fail(int code, const std::string &msg) {
  set_error(msg);
  return code;
}

int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(MTP_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  count_launch();
  return MTP_OK;
}

bool pdl_enabled() {
  static int on = -1;
  if (on < 0) {
    const char *e = getenv("MTP_PDL");
    on = (e && e[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

int num_sms() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// ----------------------------------------------------------------- kernels
template <typename T>
__global__ void embedding_kernel(const int64_t *__restrict__ ids, const T *__restrict__ table, int D,
                                 float *__restrict__ out) {
  MTP_PDL_WAIT();
  MTP_PDL_TRIGGER();
  const int t = blockIdx.x;
  const T *row = table + (size_t)ids[t] * D;
  for (int i = threadIdx.x; i < D; i += blockDim.x) out[(size_t)t * D + i] = ldf(row + i);
}

__device__ __forceinline__ float block_sum(float v, float *red) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < nw; ++i) s += red[i];  // fixed order: identical in every block
  return s;
}

template <typename TW, typename TO>
__global__ void rmsnorm_kernel(const float *__restrict__ x, int D, const TW *__restrict__ w, float eps,
                               TO *__restrict__ out) {
  MTP_PDL_WAIT();
  MTP_PDL_TRIGGER();
  __shared__ float red[32];
  const float *row = x + (size_t)blockIdx.x * D;
  float ss = 0.f;
  for (int i = threadIdx.x; i < D; i += blockDim.x) ss += row[i] * row[i];
  ss = block_sum(ss, red);
  const float r = rsqrtf(ss / (float)D + eps);
  for (int i = threadIdx.x; i < D; i += blockDim.x)
    stf(out + (size_t)blockIdx.x * D + i, ldf(w + i) * (row[i] * r));
}

template <typename T>
__global__ void argmax_kernel(const T *__restrict__ logits, int V, int ld, int64_t *__restrict__ out) {
  MTP_PDL_WAIT();
  MTP_PDL_TRIGGER();
  __shared__ float bv[32];
  __shared__ int bi[32];
  const T *row = logits + (size_t)blockIdx.x * ld;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    float v = ldf(row + i);
    if (v > best) { best = v; idx = i; }  // strided scan keeps the first index on ties
  }
  for (int o = 16; o; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, best, o);
    int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > best || (ov == best && oi < idx)) { best = ov; idx = oi; }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) { bv[w] = best; bi[w] = idx; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i)
      if (bv[i] > best || (bv[i] == best && bi[i] < idx)) { best = bv[i]; idx = bi[i]; }
    out[blockIdx.x] = idx;
  }
}

}  // namespace mtp

using namespace mtp;

extern "C" {

const char *mtp_version(void) { return "mtp 0.1 sm_100a"; }
const char *mtp_last_error(void) { return t_last_error.c_str(); }
uint64_t mtp_launch_count(void) { return g_launches.load(); }

int mtp_embedding(const int64_t *ids, int T, const void *table, int D, int dtype, float *out, void *stream) {
  MTP_REQUIRE(T >= 0 && D > 0 && ids && table && out, "bad arguments");
  if (T == 0) return MTP_OK;
  cudaStream_t s = (cudaStream_t)stream;
  MTP_DISPATCH_FB(dtype, TT, launch_pdl(embedding_kernel<TT>, dim3(T), dim3(256), 0, s, ids, (const TT *)table, D, out));
  return check_launch("embedding");
}

int mtp_rmsnorm(const float *x, int T, int D, const void *w, int w_dtype, float eps, void *out, int out_dtype,
                void *stream) {
  MTP_REQUIRE(T >= 0 && D > 0 && x && w && out, "bad arguments");
  if (T == 0) return MTP_OK;
  cudaStream_t s = (cudaStream_t)stream;
  MTP_DISPATCH_FB(w_dtype, TW, MTP_DISPATCH_FB(out_dtype, TO,
      launch_pdl(rmsnorm_kernel<TW, TO>, dim3(T), dim3(256), 0, s, x, D, (const TW *)w, eps, (TO *)out)));
  return check_launch("rmsnorm");
}

int mtp_argmax_rows(const void *logits, int T, int V, int ld, int dtype, int64_t *out, void *stream) {
  MTP_REQUIRE(T >= 0 && V > 0 && ld >= V && logits && out, "bad arguments");
  if (T == 0) return MTP_OK;
  cudaStream_t s = (cudaStream_t)stream;
  MTP_DISPATCH_FB(dtype, TT, launch_pdl(argmax_kernel<TT>, dim3(T), dim3(512), 0, s, (const TT *)logits, V, ld, out));
  return check_launch("argmax");
}

}  // extern "C"
