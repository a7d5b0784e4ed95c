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

template <typename TIn>
__global__ void __launch_bounds__(1024) argmax_kernel(const TIn* __restrict__ x, int ld, int V,
                                                      int64_t* __restrict__ out_ids,
                                                      float* __restrict__ out_vals) {
  const int row = blockIdx.x;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = to_f(x[(size_t)row * ld + i]);
    if (v > best || (v == best && i < bi)) { best = v; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffff, best, o);
    const int oi = __shfl_xor_sync(0xffffffff, bi, o);
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) { sv[w] = best; si[w] = bi; }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x / 32;
    best = l < nw ? sv[l] : -INFINITY;
    bi = l < nw ? si[l] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffff, best, o);
      const int oi = __shfl_xor_sync(0xffffffff, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (l == 0) {
      out_ids[row] = bi;
      if (out_vals) out_vals[row] = best;
    }
  }
}

// one warp per row; K <= 1024 candidates, sorted descending
__global__ void sample_topk_kernel(const float* __restrict__ vals, const int64_t* __restrict__ ids,
                                   int K, const float* __restrict__ temperature,
                                   const int* __restrict__ top_k, const float* __restrict__ top_p,
                                   const float* __restrict__ min_p, const int64_t* __restrict__ seeds,
                                   int64_t step, int64_t* __restrict__ out, float* __restrict__ out_logprob,
                                   float* __restrict__ probs_out, int B) {
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

void argmax_rows(torch::Tensor x, torch::Tensor out_ids, torch::Tensor out_vals) {
  const int B = x.size(0), V = x.size(1);
  if (B == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  float* vp = out_vals.defined() && out_vals.numel() ? out_vals.data_ptr<float>() : nullptr;
  if (x.scalar_type() == at::kFloat)
    smp::argmax_kernel<float><<<B, 1024, 0, stream>>>(x.data_ptr<float>(), x.stride(0), V,
                                                      out_ids.data_ptr<int64_t>(), vp);
  else
    smp::argmax_kernel<__nv_bfloat16><<<B, 1024, 0, stream>>>(
        (const __nv_bfloat16*)x.data_ptr(), x.stride(0), V, out_ids.data_ptr<int64_t>(), vp);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void sample_from_topk(torch::Tensor vals, torch::Tensor ids, torch::Tensor temperature,
                      torch::Tensor top_k, torch::Tensor top_p, torch::Tensor min_p,
                      torch::Tensor seeds, int64_t step, torch::Tensor out, torch::Tensor out_logprob,
                      torch::Tensor probs_out) {
  const int B = vals.size(0), K = vals.size(1);
  if (B == 0) return;
  const at::cuda::CUDAGuard guard(vals.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  smp::sample_topk_kernel<<<(B + 7) / 8, 256, 0, stream>>>(
      vals.data_ptr<float>(), ids.data_ptr<int64_t>(), K, temperature.data_ptr<float>(),
      top_k.data_ptr<int>(), top_p.data_ptr<float>(),
      min_p.defined() && min_p.numel() ? min_p.data_ptr<float>() : nullptr, seeds.data_ptr<int64_t>(),
      step, out.data_ptr<int64_t>(),
      out_logprob.defined() && out_logprob.numel() ? out_logprob.data_ptr<float>() : nullptr,
      probs_out.defined() && probs_out.numel() ? probs_out.data_ptr<float>() : nullptr, B);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace rad
