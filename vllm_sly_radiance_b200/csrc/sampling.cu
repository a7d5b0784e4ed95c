// Token sampling kernels.
//
// Reference behaviour: the sampler the reference configures (temperature / top-k / top-p /
// min-p, radiance_topk.py:1-59 "exact top-k/top-p via a top-k window") and the greedy path.
//  * argmax_rows      : one CTA per row, greedy token (ties -> lowest index).
//  * sample_from_topk : rows given as a top-K window (values + ids, sorted descending); applies
//                       temperature, top-k, top-p (nucleus, kept while the mass before a token is
//                       < p), min-p, then draws with a per-row Philox stream keyed by (seed, step).
//  * topk_window      : the top-64 window of each row (radix select per chunk, last-CTA merge),
//                       optionally followed in the same launch by the draw above.
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

// One warp draws one row from a window v[0..K) sorted descending (any memory space); id(i) gives
// the token id of window entry i.  Temperature, top-k, top-p (kept while the mass before a
// token is < p), min-p, then an inverse-CDF draw with one Philox uniform keyed by (seed, step).
template <typename IdF>
DEVI void sample_row_warp(const float* v, int K, IdF id, float T, int topk, float p, float mp,
                          int64_t seed, int64_t step, int64_t* out, float* out_logprob,
                          float* probs_out) {
  const int lane = threadIdx.x % 32;
  const int kk = topk > 0 ? min(topk, K) : K;
  if (T <= 0.f) {   // greedy
    if (lane == 0) {
      *out = id(0);
      if (out_logprob) *out_logprob = 0.f;
    }
    if (probs_out)
      for (int i = lane; i < K; i += 32) probs_out[i] = i == 0 ? 1.f : 0.f;
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
    curand_init((unsigned long long)seed, (unsigned long long)step, 0, &st);
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
    for (int i = lane; i < K; i += 32) probs_out[i] = i < keep ? __expf(v[i] / T - vmax) / zk : 0.f;
  }
  if (lane == 0) {
    *out = id(chosen);
    if (out_logprob) *out_logprob = (v[chosen] / T - vmax) - __logf(zk);
  }
}

// one warp per row; rows given as a window of K candidates sorted descending (K up to the full
// vocabulary: the full-vocabulary path hands in a sorted row)
__global__ void sample_topk_kernel(const float* __restrict__ vals, const int64_t* __restrict__ ids,
                                   int K, const float* __restrict__ temperature,
                                   const int* __restrict__ top_k, const float* __restrict__ top_p,
                                   const float* __restrict__ min_p, const int64_t* __restrict__ seeds,
                                   int64_t step, int64_t* __restrict__ out, float* __restrict__ out_logprob,
                                   float* __restrict__ probs_out, int B) {
  pdl_wait();     // inputs come from the preceding kernel
  pdl_trigger();
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (row >= B) return;
  const int64_t* rid = ids + (size_t)row * K;
  sample_row_warp(vals + (size_t)row * K, K, [&](int i) { return rid[i]; }, temperature[row],
                  top_k[row], top_p[row], min_p ? min_p[row] : 0.f, seeds[row], step, out + row,
                  out_logprob ? out_logprob + row : nullptr,
                  probs_out ? probs_out + (size_t)row * K : nullptr);
}

// ---------------------------------------------------------------------------------------------
// Top-64 window of long rows (the sampler's candidate set), no sort of the row:
//  * each CTA takes a chunk of <= 4096 logits into shared memory as order-preserving 32-bit
//    keys, finds the 64th largest key by a 4-pass radix select (8-bit digits, per-warp
//    histograms with match_any aggregation), collects the 64 winners in index order (ties at
//    the threshold go to the lowest indices) and rank-sorts them;
//  * the last CTA of the row (self-resetting arrival counter) runs the same selection over the
//    chunks' 64-candidate lists, writes the sorted window and, when sampling parameters are
//    given, draws the row's token from it with one warp.
// Reference behaviour: the composite top-k/top-p sampler of radiance_topk.py:1-59 (top-k window
// first, exact whenever every row's top_k fits in the window).
// ---------------------------------------------------------------------------------------------
constexpr int TK = 64;
constexpr int TK_CHUNK = 4096;
constexpr int TK_THREADS = 256;
constexpr int TK_WARPS = TK_THREADS / 32;

DEVI uint32_t f2key(float f) {
  if (f != f) f = -INFINITY;                    // NaN ranks last
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
DEVI float key2f(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

struct TkSmem {
  uint32_t keys[TK_CHUNK];
  int idx[TK_CHUNK];                 // merge stage: column of each candidate
  int hist[TK_WARPS][256];
  int tot[256];
  uint32_t sel_key[TK];
  int sel_idx[TK];
  float win_val[TK];
  int wtot[2][TK_WARPS];
  int sh_bin, sh_k, sh_cnt;
  uint32_t sh_thr;
  bool last;
};

// The top K of keys[0, n) (n >= K) as a digit prefix: every key whose masked value is above
// `prefix` is selected, and the first `need_eq` keys (in index order) whose masked value equals
// it.  8-bit digits from the top; the passes stop as soon as the threshold bin holds exactly the
// keys still needed (then all of them are selected).
DEVI void radix_kth(TkSmem& s, int n, int K, uint32_t& prefix_out, uint32_t& mask_out, int& need_eq) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint32_t prefix = 0, mask = 0;
  int k = K;
#pragma unroll 1
  for (int shift = 24; shift >= 0; shift -= 8) {
    int* h = &s.hist[0][0];
    for (int i = tid; i < TK_WARPS * 256; i += TK_THREADS) h[i] = 0;
    __syncthreads();
    for (int i0 = 0; i0 < n; i0 += TK_THREADS) {
      const int i = i0 + tid;
      const uint32_t u = i < n ? s.keys[i] : 0u;
      const bool act = i < n && (u & mask) == prefix;
      const uint32_t bin = (u >> shift) & 255u;
      const unsigned am = __ballot_sync(0xffffffffu, act);
      if (act) {
        const unsigned peers = __match_any_sync(am, bin);
        if (lane == __ffs(peers) - 1) atomicAdd(&s.hist[warp][bin], __popc(peers));
      }
    }
    __syncthreads();
    {   // per-bin totals: one bin per thread
      int v = 0;
#pragma unroll
      for (int w = 0; w < TK_WARPS; ++w) v += s.hist[w][tid];
      s.tot[tid] = v;
    }
    __syncthreads();
    if (warp == 0) {
      // lane l owns the bins 255 - 8l ... 248 - 8l (descending order)
      int c[8];
      int tot = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = s.tot[255 - (8 * lane + j)];
        tot += c[j];
      }
      int incl = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      const int before = incl - tot;
      if (before < k && k <= incl) {
        int cum = before;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (cum + c[j] >= k) {
            s.sh_bin = 255 - (8 * lane + j);
            s.sh_k = k - cum;
            s.sh_cnt = c[j];
            break;
          }
          cum += c[j];
        }
      }
    }
    __syncthreads();
    prefix |= (uint32_t)s.sh_bin << shift;
    mask |= 255u << shift;
    k = s.sh_k;
    if (s.sh_cnt == k) break;       // the whole bin is selected: the prefix decides
  }
  prefix_out = prefix;
  mask_out = mask;
  need_eq = k;
}

// The K selected entries in index order: every key with (key & mask) > prefix, then the first
// need_eq keys with (key & mask) == prefix.
template <typename F>
DEVI void collect_topk(TkSmem& s, int n, int K, uint32_t prefix, uint32_t mask, int need_eq, F col) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_gt = K - need_eq;
  int base_gt = 0, base_eq = 0;
  const unsigned lt = (1u << lane) - 1u;
  for (int i0 = 0; i0 < n; i0 += TK_THREADS) {
    const int i = i0 + tid;
    const uint32_t u = i < n ? s.keys[i] : 0u;
    const uint32_t um = u & mask;
    const bool gt = i < n && um > prefix;
    const bool eq = i < n && um == prefix;
    const unsigned mg = __ballot_sync(0xffffffffu, gt), me = __ballot_sync(0xffffffffu, eq);
    if (lane == 0) {
      s.wtot[0][warp] = __popc(mg);
      s.wtot[1][warp] = __popc(me);
    }
    __syncthreads();
    int pg = base_gt, pe = base_eq, tg = 0, te = 0;
#pragma unroll
    for (int w = 0; w < TK_WARPS; ++w) {
      if (w < warp) { pg += s.wtot[0][w]; pe += s.wtot[1][w]; }
      tg += s.wtot[0][w];
      te += s.wtot[1][w];
    }
    pg += __popc(mg & lt);
    pe += __popc(me & lt);
    if (gt) { s.sel_key[pg] = u; s.sel_idx[pg] = col(i); }
    if (eq && pe < need_eq) { s.sel_key[n_gt + pe] = u; s.sel_idx[n_gt + pe] = col(i); }
    base_gt += tg;
    base_eq += te;
    __syncthreads();
    if (base_gt >= n_gt && base_eq >= need_eq) break;     // uniform: every slot is filled
  }
}

// rank sort of the K selected entries: key descending, column ascending among equal keys
DEVI void rank_sort(const TkSmem& s, int K, uint32_t* out_key, int* out_idx) {
  if (threadIdx.x < K) {
    const uint32_t mk = s.sel_key[threadIdx.x];
    const int mi = s.sel_idx[threadIdx.x];
    int r = 0;
    for (int j = 0; j < K; ++j) {
      const uint32_t kj = s.sel_key[j];
      r += (kj > mk) || (kj == mk && s.sel_idx[j] < mi);
    }
    out_key[r] = mk;
    out_idx[r] = mi;
  }
}

template <typename TIn>
__global__ void __launch_bounds__(TK_THREADS) topk_window_kernel(
    const TIn* __restrict__ x, int ld, int V, int chunk, uint32_t* __restrict__ pk,
    int* __restrict__ pi, unsigned* __restrict__ counters, float* __restrict__ out_vals,
    int64_t* __restrict__ out_ids, const float* __restrict__ temperature,
    const int* __restrict__ top_k, const float* __restrict__ top_p, const float* __restrict__ min_p,
    const int64_t* __restrict__ seeds, int64_t step, int64_t* __restrict__ out_tok,
    float* __restrict__ probs_out) {
  pdl_wait();     // the logits come from the preceding kernel
  pdl_trigger();
  __shared__ TkSmem s;
  const int row = blockIdx.y, ch = blockIdx.x, nch = gridDim.x;
  const int c0 = ch * chunk;
  const int n = min(V, c0 + chunk) - c0;
  const TIn* xr = x + (size_t)row * ld + c0;
  for (int i = threadIdx.x; i < n; i += TK_THREADS) s.keys[i] = f2key(to_f(xr[i]));
  __syncthreads();
  uint32_t pre, msk;
  int need;
  radix_kth(s, n, TK, pre, msk, need);
  collect_topk(s, n, TK, pre, msk, need, [&](int i) { return c0 + i; });
  const size_t off = ((size_t)row * nch + ch) * TK;
  rank_sort(s, TK, pk + off, pi + off);
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s.last = atomicAdd(&counters[row], 1u) == (unsigned)(nch - 1);
  __syncthreads();
  if (!s.last) return;
  __threadfence();
  // merge.  Chunk c holds 64 keys >= its 64th key t_c, so the row's top 64 are all >= T* = max
  // t_c: only list entries >= T* are candidates (usually a few more than 64).  The lists are in
  // column order, so ties keep the lowest columns.
  const int nc = nch * TK;
  const uint32_t* rk = pk + (size_t)row * nc;
  const int* ri = pi + (size_t)row * nc;
  if (threadIdx.x < 32) {
    uint32_t t = 0;
    for (int c = threadIdx.x; c < nch; c += 32) t = max(t, __ldcg(rk + (size_t)c * TK + TK - 1));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t = max(t, __shfl_xor_sync(0xffffffffu, t, o));
    if (threadIdx.x == 0) { s.sh_thr = t; s.sh_cnt = 0; }
  }
  __syncthreads();
  const uint32_t tstar = s.sh_thr;
  for (int i0 = 0; i0 < nc; i0 += TK_THREADS) {     // ordered compaction of the candidates
    const int i = i0 + threadIdx.x;
    const uint32_t u = i < nc ? __ldcg(rk + i) : 0u;
    const bool keep = i < nc && u >= tstar;
    const unsigned m = __ballot_sync(0xffffffffu, keep);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) s.wtot[0][warp] = __popc(m);
    __syncthreads();
    int pos = s.sh_cnt, tot = 0;
#pragma unroll
    for (int w = 0; w < TK_WARPS; ++w) {
      if (w < warp) pos += s.wtot[0][w];
      tot += s.wtot[0][w];
    }
    pos += __popc(m & ((1u << lane) - 1u));
    if (keep) { s.keys[pos] = u; s.idx[pos] = __ldcg(ri + i); }
    __syncthreads();
    if (threadIdx.x == 0) s.sh_cnt += tot;
    __syncthreads();
  }
  const int ncand = s.sh_cnt;
  radix_kth(s, ncand, TK, pre, msk, need);
  collect_topk(s, ncand, TK, pre, msk, need, [&](int i) { return s.idx[i]; });
  rank_sort(s, TK, s.keys, s.idx);
  __syncthreads();
  if (threadIdx.x < TK) {
    const float v = key2f(s.keys[threadIdx.x]);
    s.win_val[threadIdx.x] = v;
    if (out_vals) out_vals[(size_t)row * TK + threadIdx.x] = v;
    if (out_ids) out_ids[(size_t)row * TK + threadIdx.x] = s.idx[threadIdx.x];
  }
  if (threadIdx.x == 0) counters[row] = 0;
  __syncthreads();
  if (temperature != nullptr && threadIdx.x < 32)
    sample_row_warp(s.win_val, TK, [&](int i) { return (int64_t)s.idx[i]; }, temperature[row],
                    top_k[row], top_p[row], min_p ? min_p[row] : 0.f, seeds[row], step,
                    out_tok + row, nullptr, probs_out ? probs_out + (size_t)row * TK : nullptr);
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

// Top-64 window of each row of x [B, V] (bf16 or fp32), V <= 64 * 4096.  workspace: int32, fixed
// layout [0, 4096) arrival counters (zero, self-resetting), then per-row chunk candidate keys and
// columns (B * 64 * 64 each).  With sampling parameters (temperature defined) the last CTA of each
// row also draws the row's token into out_tok (and the window probabilities into probs_out).
void topk_window(torch::Tensor x, torch::Tensor out_vals, torch::Tensor out_ids,
                 torch::Tensor workspace, torch::Tensor temperature, torch::Tensor top_k,
                 torch::Tensor top_p, torch::Tensor min_p, torch::Tensor seeds, int64_t step,
                 torch::Tensor out_tok, torch::Tensor probs_out) {
  using namespace smp;
  const int B = x.size(0), V = x.size(1);
  if (B == 0) return;
  TORCH_CHECK(x.stride(1) == 1, "topk_window: rows must be contiguous");
  TORCH_CHECK(V >= TK && V <= 64 * TK_CHUNK, "topk_window: 64 <= vocab <= 262144");
  TORCH_CHECK(B <= 4096, "topk_window: at most 4096 rows");
  const int nch = (V + TK_CHUNK - 1) / TK_CHUNK;
  const int chunk = (V + nch - 1) / nch;
  TORCH_CHECK(workspace.numel() >= 4096 + (int64_t)B * nch * TK * 2, "topk_window: workspace too small");
  const at::cuda::CUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  unsigned* cnt = reinterpret_cast<unsigned*>(workspace.data_ptr());
  uint32_t* pk = reinterpret_cast<uint32_t*>(cnt + 4096);
  int* pi = reinterpret_cast<int*>(pk + (size_t)B * nch * TK);
  const bool draw = temperature.defined() && temperature.numel();
  auto fp = [](const torch::Tensor& t) { return t.defined() && t.numel() ? t.data_ptr<float>() : nullptr; };
  const float* tp = draw ? temperature.data_ptr<float>() : nullptr;
  const int* tk = draw ? top_k.data_ptr<int>() : nullptr;
  const float* pp = draw ? top_p.data_ptr<float>() : nullptr;
  const float* mp = draw ? fp(min_p) : nullptr;
  const int64_t* sd = draw ? seeds.data_ptr<int64_t>() : nullptr;
  int64_t* ot = draw ? out_tok.data_ptr<int64_t>() : nullptr;
  float* pr = draw ? fp(probs_out) : nullptr;
  float* ov = fp(out_vals);
  int64_t* oi = out_ids.defined() && out_ids.numel() ? out_ids.data_ptr<int64_t>() : nullptr;
  dim3 grid(nch, B);
  if (x.scalar_type() == at::kFloat)
    C10_CUDA_CHECK(launch_pdl((topk_window_kernel<float>), grid, dim3(TK_THREADS), 0, stream,
                              x.data_ptr<float>(), (int)x.stride(0), V, chunk, pk, pi, cnt, ov, oi,
                              tp, tk, pp, mp, sd, step, ot, pr));
  else {
    TORCH_CHECK(x.scalar_type() == at::kBFloat16, "topk_window: bf16 or fp32 logits");
    C10_CUDA_CHECK(launch_pdl((topk_window_kernel<__nv_bfloat16>), grid, dim3(TK_THREADS), 0, stream,
                              (const __nv_bfloat16*)x.data_ptr(), (int)x.stride(0), V, chunk, pk, pi,
                              cnt, ov, oi, tp, tk, pp, mp, sd, step, ot, pr));
  }
}

}  // namespace rad
