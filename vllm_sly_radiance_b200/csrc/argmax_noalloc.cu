// Greedy argmax over logits rows through a C entry point that allocates no device memory.
//
// This entry point has no counterpart in the reference, whose greedy path always runs inside
// PyTorch and takes its temporaries from the caching allocator.  It exists for callers that
// cannot allocate at the moment they need a token:
//   * a host runtime written in C or C++ that links this library without torch, and so has no
//     caching allocator to draw a workspace from;
//   * a serving process after the KV cache has been sized to take nearly all free HBM, where a
//     late cudaMalloc may fail outright;
//   * a latency-bound decode loop, where cudaMalloc / cudaFree may synchronise the whole device
//     and stall every stream that is in flight.
//
// The kernel is the multi-CTA argmax of sampling.cu in a form that takes its partials and arrival
// counters from one file-scope __device__ array (`g_argmax_scratch`, about 516 KB per device)
// instead of a caller workspace.  Limits: at most kNoAllocMaxRows rows per call and at most
// kNoAllocMaxChunks CTAs per row (the vocabulary is split into that many chunks at most, so any
// vocabulary size fits).  Calls outside those limits are rejected with an error message; nothing
// is launched.
//
// Set-up: the first call in each CUDA context (the runtime's primary context of a device, or a
// context the caller created with the driver API), with that context current, resolves the
// scratch address with cudaGetSymbolAddress and caches it for that context: a device address is
// only valid in the context it was resolved in.  Make that first call before any stream capture
// begins.  The C declaration and the limits are in radiance_noalloc.h; the file is built both
// into the torch extension and, alone, into libradiance_noalloc.so, which links only the CUDA
// runtime.
//
// Concurrency: the scratch is one per device, so calls that overlap on the same device (two host
// threads, or two streams whose launches run at the same time) race on it and may return wrong
// tokens.  Serialise calls per device, e.g. by issuing them all on one stream.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>
#include <stdio.h>

#include <mutex>

#include "radiance_noalloc.h"

namespace rad {
namespace noalloc {

constexpr int kNoAllocMaxRows = RADIANCE_NOALLOC_MAX_ROWS;
constexpr int kNoAllocMaxChunks = RADIANCE_NOALLOC_MAX_CHUNKS;
constexpr int kMaxContexts = RADIANCE_NOALLOC_MAX_CONTEXTS;
constexpr int kThreads = 256;

struct ArgmaxScratch {
  unsigned counters[kNoAllocMaxRows];                        // must be zero when a call starts
  float part_val[kNoAllocMaxRows * kNoAllocMaxChunks];
  int part_idx[kNoAllocMaxRows * kNoAllocMaxChunks];
};

static __device__ __align__(256) ArgmaxScratch g_argmax_scratch;

__device__ __forceinline__ float load_f(const float* p) { return *p; }
__device__ __forceinline__ float load_f(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// larger value wins; equal values -> lower index
__device__ __forceinline__ void better(float& v, int& i, float ov, int oi) {
  if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
}

__device__ __forceinline__ void cta_reduce(float& v, int& i, float* sv, int* si) {
  for (int o = 16; o > 0; o >>= 1)
    better(v, i, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, i, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) { sv[warp] = v; si[warp] = i; }
  __syncthreads();
  v = lane < (int)(blockDim.x >> 5) ? sv[lane] : -INFINITY;
  i = lane < (int)(blockDim.x >> 5) ? si[lane] : 0x7fffffff;
  for (int o = 16; o > 0; o >>= 1)
    better(v, i, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, i, o));
}

// grid (chunks, rows): each CTA reduces one chunk of one row to a partial (value, index); the
// CTA that arrives last on the row's counter reduces the row's partials and clears the counter.
template <typename T>
__global__ void __launch_bounds__(kThreads) argmax_static_kernel(
    const T* __restrict__ x, long long ld, int vocab, int chunk, ArgmaxScratch* __restrict__ s,
    long long* __restrict__ out_ids, float* __restrict__ out_vals) {
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ bool is_last;
  const int row = blockIdx.y, ch = blockIdx.x, nch = gridDim.x;
  const T* xr = x + (size_t)row * (size_t)ld;
  float v = -INFINITY;
  int i = 0x7fffffff;
  const int c0 = ch * chunk, c1 = min(vocab, c0 + chunk);
  for (int j = c0 + (int)threadIdx.x; j < c1; j += kThreads) better(v, i, load_f(xr + j), j);
  cta_reduce(v, i, sv, si);
  const int slot = row * kNoAllocMaxChunks + ch;
  if (threadIdx.x == 0) {
    s->part_val[slot] = v;
    s->part_idx[slot] = i;
    __threadfence();
    is_last = atomicAdd(&s->counters[row], 1u) == (unsigned)(nch - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  v = -INFINITY;
  i = 0x7fffffff;
  const volatile float* pv = s->part_val + row * kNoAllocMaxChunks;
  const volatile int* pi = s->part_idx + row * kNoAllocMaxChunks;
  for (int c = threadIdx.x; c < nch; c += kThreads) better(v, i, pv[c], pi[c]);
  cta_reduce(v, i, sv, si);
  if (threadIdx.x == 0) {
    out_ids[row] = i;
    if (out_vals) out_vals[row] = v;
    s->counters[row] = 0;
  }
}

// scratch address per CUDA context (fixed table: the set-up allocates nothing, host or device)
std::mutex g_setup_mu;
CUcontext g_ctx[kMaxContexts] = {};
ArgmaxScratch* g_ctx_scratch[kMaxContexts] = {};
int g_num_ctx = 0;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

// the current context through the runtime's driver entry-point query (no link to libcuda)
cudaError_t current_context(CUcontext* ctx) {
  static CtxGetCurrentFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess) return e;
    if (q != cudaDriverEntryPointSuccess || !p) return cudaErrorNotSupported;
    fn = reinterpret_cast<CtxGetCurrentFn>(p);
  }
  return fn(ctx) == CUDA_SUCCESS ? cudaSuccess : cudaErrorContextIsDestroyed;
}

int fail(char* err, int err_len, int code, const char* msg) {
  if (err && err_len > 0) snprintf(err, (size_t)err_len, "%s", msg);
  return code;
}

}  // namespace noalloc
}  // namespace rad

// Declared in radiance_noalloc.h.  Returns 0 on success.  On failure returns a nonzero code (a
// cudaError_t value for CUDA failures, -1 for a rejected argument) and writes a message into
// err[0:err_len) when err is non-null.
//   logits   : device pointer, rows x vocab, row stride ld elements; dtype 0 = bf16, 1 = fp32
//   out_ids  : device int64 [rows]; out_vals: device fp32 [rows] or null
//   stream   : cudaStream_t to launch on (null = legacy default stream)
extern "C" int radiance_argmax_rows_noalloc(const void* logits, int dtype, int rows, int vocab,
                                            long long ld, long long* out_ids, float* out_vals,
                                            void* stream, char* err, int err_len) {
  using namespace rad::noalloc;
  if (rows <= 0 || rows > kNoAllocMaxRows)
    return fail(err, err_len, -1, "radiance_argmax_rows_noalloc: rows must be in [1, 1024]");
  if (vocab <= 0 || ld < vocab)
    return fail(err, err_len, -1, "radiance_argmax_rows_noalloc: need vocab > 0 and ld >= vocab");
  if (dtype != 0 && dtype != 1)
    return fail(err, err_len, -1, "radiance_argmax_rows_noalloc: dtype must be 0 (bf16) or 1 (fp32)");
  if (!logits || !out_ids)
    return fail(err, err_len, -1, "radiance_argmax_rows_noalloc: null logits or out_ids");

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(err, err_len, (int)e, cudaGetErrorString(e));
  // cudaGetDevice / cudaPointerGetAttributes make the primary context current when none is
  CUcontext ctx = nullptr;
  cudaPointerAttributes attr;
  e = cudaPointerGetAttributes(&attr, logits);
  if (e != cudaSuccess) return fail(err, err_len, (int)e, cudaGetErrorString(e));
  if (attr.type != cudaMemoryTypeDevice || attr.device != dev)
    return fail(err, err_len, -1,
                "radiance_argmax_rows_noalloc: logits must be device memory of the current device");

  e = current_context(&ctx);
  if (e != cudaSuccess || !ctx)
    return fail(err, err_len, e != cudaSuccess ? (int)e : -1,
                "radiance_argmax_rows_noalloc: no current CUDA context");

  ArgmaxScratch* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    for (int c = 0; c < g_num_ctx; ++c)
      if (g_ctx[c] == ctx) scratch = g_ctx_scratch[c];
    if (!scratch) {
      if (g_num_ctx == kMaxContexts)
        return fail(err, err_len, -1, "radiance_argmax_rows_noalloc: more than 64 CUDA contexts");
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_argmax_scratch);
      if (e != cudaSuccess) return fail(err, err_len, (int)e, cudaGetErrorString(e));
      scratch = static_cast<ArgmaxScratch*>(p);
      g_ctx[g_num_ctx] = ctx;
      g_ctx_scratch[g_num_ctx] = scratch;
      ++g_num_ctx;
    }
  }

  // about 4096 logits per CTA, at most kNoAllocMaxChunks CTAs per row
  const long long want = ((long long)vocab + 4095) / 4096;
  const int nch = (int)(want < kNoAllocMaxChunks ? want : kNoAllocMaxChunks);
  const int chunk = (int)(((long long)vocab + nch - 1) / nch);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the arrival counters must read zero when the launch starts
  unsigned* counters = reinterpret_cast<unsigned*>(reinterpret_cast<char*>(scratch) +
                                                   offsetof(ArgmaxScratch, counters));
  e = cudaMemsetAsync(counters, 0, sizeof(unsigned) * (size_t)rows, st);
  if (e != cudaSuccess) return fail(err, err_len, (int)e, cudaGetErrorString(e));
  const dim3 grid(nch, rows);
  if (dtype == 0)
    argmax_static_kernel<__nv_bfloat16><<<grid, kThreads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(logits), ld, vocab, chunk, scratch, out_ids, out_vals);
  else
    argmax_static_kernel<float><<<grid, kThreads, 0, st>>>(
        static_cast<const float*>(logits), ld, vocab, chunk, scratch, out_ids, out_vals);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(err, err_len, (int)e, cudaGetErrorString(e));
  return 0;
}
