// Token sampling kernels.
//
// Reference behaviour: the sampler the reference configures (temperature / top-k / top-p /
// min-p, radiance_topk.py:1-59 "exact top-k/top-p via a top-k window") and the greedy path.
//  * argmax_rows      : one CTA per row, greedy token (ties -> lowest index).
//  * sample_from_topk : rows given as a top-K window (values + ids, sorted descending); applies
//                       temperature, top-k, top-p (nucleus, kept while the mass before a token is
//                       < p), min-p, then draws with a per-row Philox stream keyed by (seed, step).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <curand_kernel.h>
#include <torch/extension.h>

#include "common.cuh"

namespace rad {
namespace smp {

// Greedy argmax over long rows, split across CTAs: each CTA reduces one chunk of a row to
// (value, index); the last CTA of the row (self-resetting arrival counter) reduces the partials.
// Ties resolve to the lowest index.
DEVI void argmax_combine(float& best, int& bi, float ov, int oi) {
  if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
}
DEVI void block_argmax(float& best, int& bi, float* sv, int* si) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    argmax_combine(best, bi, __shfl_xor_sync(0xffffffff, best, o), __shfl_xor_sync(0xffffffff, bi, o));
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  __syncthreads();
  if (l == 0) { sv[w] = best; si[w] = bi; }
  __syncthreads();
  const int nw = blockDim.x / 32;
  best = l < nw ? sv[l] : -INFINITY;
  bi = l < nw ? si[l] : 0x7fffffff;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    argmax_combine(best, bi, __shfl_xor_sync(0xffffffff, best, o), __shfl_xor_sync(0xffffffff, bi, o));
}

template <typename TIn>
__global__ void __launch_bounds__(256) argmax_kernel(const TIn* __restrict__ x, int ld, int V,
                                                     int chunk, float* __restrict__ pv,
                                                     int* __restrict__ pi,
                                                     unsigned* __restrict__ counters,
                                                     int64_t* __restrict__ out_ids,
                                                     float* __restrict__ out_vals) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ bool last;
  const int row = blockIdx.y, ch = blockIdx.x, nch = gridDim.x;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  const int i0 = ch * chunk, i1 = min(V, i0 + chunk);
  for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) argmax_combine(best, bi, to_f(x[(size_t)row * ld + i]), i);
  block_argmax(best, bi, sv, si);
  if (threadIdx.x == 0) {
    pv[row * nch + ch] = best;
    pi[row * nch + ch] = bi;
    __threadfence();
    last = atomicAdd(&counters[row], 1u) == (unsigned)(nch - 1);
  }
  // (counters are per row at fixed offsets; the last CTA of the row resets its counter)
  __syncthreads();
  if (!last) return;
  __threadfence();
  best = -INFINITY;
  bi = 0x7fffffff;
  for (int c = threadIdx.x; c < nch; c += blockDim.x)
    argmax_combine(best, bi, ((volatile float*)pv)[row * nch + c], ((volatile int*)pi)[row * nch + c]);
  block_argmax(best, bi, sv, si);
  if (threadIdx.x == 0) {
    out_ids[row] = bi;
    if (out_vals) out_vals[row] = best;
    counters[row] = 0;
  }
}

// one warp per row; K <= 1024 candidates, sorted descending
__global__ void sample_topk_kernel(const float* __restrict__ vals, const int64_t* __restrict__ ids,
                                   int K, const float* __restrict__ temperature,
                                   const int* __restrict__ top_k, const float* __restrict__ top_p,
                                   const float* __restrict__ min_p, const int64_t* __restrict__ seeds,
                                   int64_t step, int64_t* __restrict__ out, float* __restrict__ out_logprob,
                                   float* __restrict__ probs_out, int B) {
  pdl_wait();     // inputs come from the preceding kernel
  pdl_trigger();
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= B) return;
  const float* v = vals + (size_t)row * K;
  const float T = temperature[row];
  const int kk = top_k[row] > 0 ? min(top_k[row], K) : K;
  const float p = top_p[row];
  const float mp = min_p ? min_p[row] : 0.f;
  if (T <= 0.f) {   // greedy
    if (lane == 0) {
      out[row] = ids[(size_t)row * K];
      if (out_logprob) out_logprob[row] = 0.f;
    }
    return;
  }
  const float vmax = v[0] / T;
  // softmax denominator over the top-k window
  float z = 0.f;
  for (int i = lane; i < kk; i += 32) z += __expf(v[i] / T - vmax);
  z = warp_sum(z);
  // top-p / min-p cut: keep i while cumulative mass before i < p (and prob >= min_p * p_max)
  // the window is sorted, so the cut is a prefix; find its length with a warp scan
  int keep = kk;
  float cum = 0.f;
  for (int base = 0; base < kk; base += 32) {
    const int i = base + lane;
    float pi = i < kk ? __expf(v[i] / T - vmax) / z : 0.f;
    // inclusive scan
    float s = pi;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float t = __shfl_up_sync(0xffffffff, s, o);
      if (lane >= o) s += t;
    }
    const float before = cum + s - pi;
    const bool drop = (i < kk) && i > 0 && (before >= p || pi < mp * (1.f / z));
    const unsigned m = __ballot_sync(0xffffffff, drop);
    if (m) { keep = base + __ffs(m) - 1; break; }
    cum += __shfl_sync(0xffffffff, s, 31);
  }
  // renormalised draw over the kept prefix (inverse CDF with one Philox uniform)
  float zk = 0.f;
  for (int i = lane; i < keep; i += 32) zk += __expf(v[i] / T - vmax);
  zk = warp_sum(zk);
  float u = 0.f;
  if (lane == 0) {
    curandStatePhilox4_32_10_t st;
    curand_init((unsigned long long)seeds[row], (unsigned long long)step, 0, &st);
    u = curand_uniform(&st) * zk;
  }
  u = __shfl_sync(0xffffffff, u, 0);
  int chosen = keep - 1;
  float acc = 0.f;
  for (int base = 0; base < keep; base += 32) {
    const int i = base + lane;
    const float e = i < keep ? __expf(v[i] / T - vmax) : 0.f;
    float s = e;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float t = __shfl_up_sync(0xffffffff, s, o);
      if (lane >= o) s += t;
    }
    const bool hit = (i < keep) && (acc + s >= u);
    const unsigned m = __ballot_sync(0xffffffff, hit);
    if (m) { chosen = base + __ffs(m) - 1; break; }
    acc += __shfl_sync(0xffffffff, s, 31);
  }
  if (probs_out) {
    for (int i = lane; i < K; i += 32)
      probs_out[(size_t)row * K + i] = i < keep ? __expf(v[i] / T - vmax) / zk : 0.f;
  }
  if (lane == 0) {
    out[row] = ids[(size_t)row * K + chosen];
    if (out_logprob) out_logprob[row] = (v[chosen] / T - vmax) - __logf(zk);
  }
}

}  // namespace smp

// workspace: float[B*64] values, int[B*64] indices, uint32 counters[B] (zero, self-resetting)
void argmax_rows(torch::Tensor x, torch::Tensor out_ids, torch::Tensor out_vals,
                 torch::Tensor workspace) {
  const int B = x.size(0), V = x.size(1);
  if (B == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  float* vp = out_vals.defined() && out_vals.numel() ? out_vals.data_ptr<float>() : nullptr;
  const int nch = std::max(1, std::min(64, (V + 4095) / 4096));
  const int chunk = (V + nch - 1) / nch;
  // fixed layout independent of B (counters must stay zero between launches of any batch size):
  // [0, 4096) arrival counters, then values and indices of up to 64 chunks per row
  TORCH_CHECK(B <= 4096 && workspace.numel() >= 4096 + (int64_t)B * 64 * 2, "argmax workspace too small");
  unsigned* cnt = reinterpret_cast<unsigned*>(workspace.data_ptr());
  float* pv = reinterpret_cast<float*>(cnt + 4096);
  int* pi = reinterpret_cast<int*>(pv + B * 64);
  dim3 grid(nch, B);
  if (x.scalar_type() == at::kFloat)
    C10_CUDA_CHECK(launch_pdl((smp::argmax_kernel<float>), grid, dim3(256), 0, stream,
                              x.data_ptr<float>(), (int)x.stride(0), V, chunk, pv, pi, cnt,
                              out_ids.data_ptr<int64_t>(), vp));
  else
    C10_CUDA_CHECK(launch_pdl((smp::argmax_kernel<__nv_bfloat16>), grid, dim3(256), 0, stream,
                              (const __nv_bfloat16*)x.data_ptr(), (int)x.stride(0), V, chunk, pv,
                              pi, cnt, out_ids.data_ptr<int64_t>(), vp));
}

void sample_from_topk(torch::Tensor vals, torch::Tensor ids, torch::Tensor temperature,
                      torch::Tensor top_k, torch::Tensor top_p, torch::Tensor min_p,
                      torch::Tensor seeds, int64_t step, torch::Tensor out, torch::Tensor out_logprob,
                      torch::Tensor probs_out) {
  const int B = vals.size(0), K = vals.size(1);
  if (B == 0) return;
  const at::cuda::CUDAGuard guard(vals.device());
  auto stream = at::cuda::getCurrentCUDAStream();
C10_CUDA_CHECK(launch_pdl(  smp::sample_topk_kernel, dim3((B + 7) / 8), dim3(256), 0, stream, 
      vals.data_ptr<float>(), ids.data_ptr<int64_t>(), K, temperature.data_ptr<float>(),
      top_k.data_ptr<int>(), top_p.data_ptr<float>(),
      min_p.defined() && min_p.numel() ? min_p.data_ptr<float>() : nullptr, seeds.data_ptr<int64_t>(),
      step, out.data_ptr<int64_t>(),
      out_logprob.defined() && out_logprob.numel() ? out_logprob.data_ptr<float>() : nullptr,
      probs_out.defined() && probs_out.numel() ? probs_out.data_ptr<float>() : nullptr, B));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace rad
