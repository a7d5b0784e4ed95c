// Speculative-decoding kernels: rejection sampling with the reference's acceptance rules, and
// the prompt-lookup draft scan.
//
// Reference behaviour: vLLM's rejection sampler with sly/patch_cactus.py and sly/patch_nsd.py
// (README.md:452-578), and the lookup drafter sly/radiance_lookup_draft.py:101,129.
//
//  * rejection_kernel: one warp per request walks its k drafts in order.  Target distributions
//    arrive as the sampler's top-W windows (ids + probs, sorted descending, W <= 64: two entries
//    per lane), draft distributions as candidate windows (or a point mass on the drafted token).
//      stock (Leviathan): accept d with probability min(1, p(d) / q(d))
//      Cactus: h = clamp(p + sqrt(2 delta_eff p (1 - p)), 0, 1), capped at 1 - r (1 - p);
//              escape mixture eps runs the stock test instead (same uniform)
//      NSD: stock OR target mass strictly above p(d) <= theta
//      greedy rows: accept iff d == argmax p; on the first mismatch emit argmax p
//    On rejection a token is drawn from norm(max(0, p - q)) (p itself if that is empty); after
//    k acceptances a bonus token is drawn from p_k.  Uniforms come from a Philox stream keyed by
//    the row seed, so a seeded request reproduces its draws.
//  * lookup_kernel: one CTA per request finds the most recent earlier occurrence of the longest
//    suffix (max_ngram .. min_ngram tokens) in the request's token history and proposes the k
//    tokens that followed it.
//  * walk_kernel: the DFlash2 candidate path walk (dflash2/speculator.py:16 _selector_walk_kernel
//    behaviour).  One warp per request, one lane per candidate (Kc <= 32); step i scores the
//    candidates of draft position i against the token chosen at step i - 1 (the anchor at step
//    0): unary + sum_r pred[prev, r] * hproj[i, r] * succ[cand, r], then picks the argmax at
//    T = 0 or the Gumbel-noised argmax of score / T, and records the window probabilities
//    (softmax(score / T), one-hot at T = 0) that the rejection sampler uses as q.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <curand_kernel.h>
#include <torch/extension.h>

#include "common.cuh"

namespace rad {
namespace spec {

constexpr int kWin = 64;      // max window entries (2 per lane)

struct Rule {
  int kind;                   // 0 leviathan, 1 cactus, 2 nsd
  float delta;
  int fade_start, fade_end;
  float cap_r, escape, theta;
};

// window entry j of lane: j = lane and lane + 32
DEVI float win_lookup(const int64_t* ids, const float* pr, int W, int64_t tok, int lane) {
  float v = 0.f;
  if (lane < W && ids[lane] == tok) v += pr[lane];
  if (lane + 32 < W && ids[lane + 32] == tok) v += pr[lane + 32];
  return warp_sum(v);
}

// inverse-CDF draw over (unnormalised) weights w0 (entry lane), w1 (entry lane + 32)
DEVI int64_t win_sample(const int64_t* ids, int W, float w0, float w1, float u, int lane) {
  const float z = warp_sum(w0 + w1);
  if (!(z > 0.f)) return ids[0];
  const float target = fminf(u, 1.f - 1e-7f) * z;
  // inclusive scan of w0 over lanes, then of w1 over lanes (entries 32..63 follow 0..31)
  float c0 = w0;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float t = __shfl_up_sync(0xffffffffu, c0, o);
    if (lane >= o) c0 += t;
  }
  const float tot0 = __shfl_sync(0xffffffffu, c0, 31);
  float c1 = w1;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float t = __shfl_up_sync(0xffffffffu, c1, o);
    if (lane >= o) c1 += t;
  }
  c1 += tot0;
  // first entry whose cumulative weight exceeds the target (entries with zero weight skipped)
  const unsigned m0 = __ballot_sync(0xffffffffu, lane < W && w0 > 0.f && c0 > target);
  if (m0) return ids[__ffs(m0) - 1];
  const unsigned m1 = __ballot_sync(0xffffffffu, lane + 32 < W && w1 > 0.f && c1 > target);
  if (m1) return ids[32 + __ffs(m1) - 1];
  // rounding: the last entry with weight
  const unsigned l0 = __ballot_sync(0xffffffffu, lane < W && w0 > 0.f);
  const unsigned l1 = __ballot_sync(0xffffffffu, lane + 32 < W && w1 > 0.f);
  if (l1) return ids[32 + 31 - __clz(l1)];
  return ids[31 - __clz(l0)];
}

__global__ void rejection_kernel(const int64_t* __restrict__ draft, int k,
                                 const int64_t* __restrict__ t_ids, const float* __restrict__ t_pr,
                                 int W, const int64_t* __restrict__ d_ids,
                                 const float* __restrict__ d_pr, int Kd,
                                 const bool* __restrict__ greedy,
                                 const int64_t* __restrict__ seq_lens,
                                 const int64_t* __restrict__ forced,
                                 const int64_t* __restrict__ seeds, Rule rule, int B,
                                 int64_t* __restrict__ out, int64_t* __restrict__ n_acc) {
  pdl_wait();     // windows come from the preceding kernels
  pdl_trigger();
  const int b = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (b >= B) return;
  curandStatePhilox4_32_10_t rng;
  curand_init((unsigned long long)seeds[b], 0ull, 0ull, &rng);
  const bool g = greedy[b];
  float dlt = rule.delta;
  if (rule.kind == 1 && rule.fade_end != 0) {
    const float sl = (float)seq_lens[b];
    if (rule.fade_end <= rule.fade_start) dlt = sl >= rule.fade_start ? 0.f : dlt;
    else dlt *= fminf(fmaxf((rule.fade_end - sl) / (float)(rule.fade_end - rule.fade_start), 0.f), 1.f);
  }
  int64_t* orow = out + (size_t)b * (k + 1);
  for (int i = lane; i < k + 1; i += 32) orow[i] = -1;
  __syncwarp();
  int acc_n = 0;
  for (int i = 0; i <= k; ++i) {
    const int64_t* ids = t_ids + ((size_t)b * (k + 1) + i) * W;
    const float* pr = t_pr + ((size_t)b * (k + 1) + i) * W;
    // one draw of four uniforms per position (same in every lane: identical Philox state)
    const float4 u4 = curand_uniform4(&rng);
    const float u_acc = u4.x, u_res = u4.y, u_esc = u4.z;
    const float p0 = lane < W ? pr[lane] : 0.f;
    const float p1 = lane + 32 < W ? pr[lane + 32] : 0.f;
    if (i == k) {                                   // bonus token
      const int64_t tok = g ? ids[0] : win_sample(ids, W, p0, p1, u_res, lane);
      if (lane == 0) orow[i] = tok;
      break;
    }
    const int64_t d = draft[(size_t)b * k + i];
    bool acc;
    if (forced) {
      acc = i < forced[b];
    } else if (g) {
      acc = d == ids[0];
    } else {
      const float pt = win_lookup(ids, pr, W, d, lane);
      float qd = 1.f;
      if (d_ids) {
        const int64_t* di = d_ids + ((size_t)b * k + i) * Kd;
        const float* dp = d_pr + ((size_t)b * k + i) * Kd;
        qd = win_lookup(di, dp, Kd, d, lane);
      }
      qd = fmaxf(qd, 1e-20f);
      const bool stock = u_acc < fminf(pt / qd, 1.f);
      if (rule.kind == 1) {
        float h = fminf(fmaxf(pt + sqrtf(fmaxf(2.f * dlt * pt * (1.f - pt), 0.f)), 0.f), 1.f);
        if (rule.cap_r > 0.f) h = fminf(h, 1.f - rule.cap_r * (1.f - pt));
        const bool cac = u_acc < fminf(h / qd, 1.f);
        acc = (rule.escape > 0.f && u_esc < rule.escape) ? stock : cac;
      } else if (rule.kind == 2) {
        const float higher = warp_sum((p0 > pt ? p0 : 0.f) + (p1 > pt ? p1 : 0.f));
        acc = stock || (pt > 0.f && higher <= rule.theta);
      } else {
        acc = stock;
      }
    }
    if (acc) {
      if (lane == 0) orow[i] = d;
      ++acc_n;
      continue;
    }
    int64_t tok;
    if (g || forced) {
      tok = ids[0];
    } else {
      // residual max(0, p - q) over the target window
      float q0 = 0.f, q1 = 0.f;
      if (d_ids) {
        const int64_t* di = d_ids + ((size_t)b * k + i) * Kd;
        const float* dp = d_pr + ((size_t)b * k + i) * Kd;
        for (int j = 0; j < Kd; ++j) {
          const int64_t dj = di[j];
          if (lane < W && ids[lane] == dj) q0 += dp[j];
          if (lane + 32 < W && ids[lane + 32] == dj) q1 += dp[j];
        }
      } else {
        q0 = (lane < W && ids[lane] == d) ? 1.f : 0.f;
        q1 = (lane + 32 < W && ids[lane + 32] == d) ? 1.f : 0.f;
      }
      float r0 = fmaxf(p0 - q0, 0.f), r1 = fmaxf(p1 - q1, 0.f);
      if (!(warp_sum(r0 + r1) > 0.f)) { r0 = p0; r1 = p1; }
      tok = win_sample(ids, W, r0, r1, u_res, lane);
    }
    if (lane == 0) orow[i] = tok;
    break;
  }
  if (lane == 0) n_acc[b] = acc_n;
}

// hist [rows, Lmax] int32 token histories; request b uses row rows[b] of length len[b]; proposes
// up to k tokens per request into out [B, k] (-1 padded) and the count into n_out [B].
__global__ void __launch_bounds__(256) lookup_kernel(const int* __restrict__ hist, int Lmax,
                                                     const int* __restrict__ rows,
                                                     const int* __restrict__ len, int k,
                                                     int max_ngram, int min_ngram,
                                                     int* __restrict__ out, int* __restrict__ n_out) {
  const int b = blockIdx.x;
  const int L = len[b];
  const int* h = hist + (size_t)rows[b] * Lmax;
  __shared__ int s_best;
  for (int i = threadIdx.x; i < k; i += blockDim.x) out[(size_t)b * k + i] = -1;
  int found = -1;
  for (int n = min(max_ngram, L - 1); n >= min_ngram && found < 0; --n) {
    // candidate end positions e (exclusive): h[e - n, e) == suffix, e + 1 <= L - 1 so at least
    // one continuation token exists; keep the most recent (largest e)
    if (threadIdx.x == 0) s_best = -1;
    __syncthreads();
    for (int e = L - 1 - threadIdx.x; e >= n; e -= blockDim.x) {
      bool match = true;
      for (int j = 1; j <= n && match; ++j) match = h[e - j] == h[L - j];
      if (match) atomicMax(&s_best, e);
    }
    __syncthreads();
    found = s_best;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    int cnt = 0;
    if (found >= 0)
      for (int i = 0; i < k && found + i < L; ++i) out[(size_t)b * k + cnt++] = h[found + i];
    n_out[b] = cnt;
  }
}

// one warp per request; lanes = candidates
__global__ void __launch_bounds__(128) walk_kernel(
    const float* __restrict__ unary, const int64_t* __restrict__ cand,
    const int64_t* __restrict__ anchors, const float* __restrict__ hp,
    const __nv_bfloat16* __restrict__ pred, const __nv_bfloat16* __restrict__ succ,
    const float* __restrict__ temps, const int64_t* __restrict__ seeds, int B, int k, int Kc,
    int r, int64_t V, int64_t* __restrict__ drafts, float* __restrict__ winp,
    int* __restrict__ status) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (b >= B) return;
  const float t = temps[b];
  curandStatePhilox4_32_10_t rng;
  curand_init((unsigned long long)seeds[b], 0ull, 0ull, &rng);
  int64_t prev = anchors[b];
  for (int i = 0; i < k; ++i) {
    const size_t row = ((size_t)b * k + i) * Kc;
    const bool live = lane < Kc;
    int64_t c = live ? cand[row + lane] : 0;
    if (c < 0 || c >= V) {
      if (live) atomicExch(status, (int)kErrBounds);
      c = 0;
    }
    if (prev < 0 || prev >= V) {
      if (lane == 0) atomicExch(status, (int)kErrBounds);
      prev = 0;
    }
    float sc = -INFINITY;
    if (live) {
      const __nv_bfloat16* pp = pred + (size_t)prev * r;
      const __nv_bfloat16* sp = succ + (size_t)c * r;
      const float* hv = hp + ((size_t)b * k + i) * r;
      float acc = 0.f;
      for (int j = 0; j < r; ++j)
        acc += __bfloat162float(pp[j]) * hv[j] * __bfloat162float(sp[j]);
      sc = unary[row + lane] + acc;
    }
    // greedy choice (first maximum)
    float best = sc;
    int bi = live ? lane : 32;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    int ch = bi;
    float w = live && lane == bi ? 1.f : 0.f;
    // uniforms for the Gumbel noise: ceil(Kc / 4) draws of four per step; every lane holds the
    // same Philox state and keeps the uniform of its own candidate
    float u = 0.5f;
    for (int d = 0; d < (Kc + 3) / 4; ++d) {
      const float4 v = curand_uniform4(&rng);
      if ((lane >> 2) == d) {
        const int e = lane & 3;
        u = e == 0 ? v.x : e == 1 ? v.y : e == 2 ? v.z : v.w;
      }
    }
    if (t > 0.f) {
      const float st = live ? sc / t : -INFINITY;
      float mx = st;
#pragma unroll
      for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float ex = live ? __expf(st - mx) : 0.f;
      float sum = ex;
#pragma unroll
      for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      w = ex / sum;
      u = fminf(fmaxf(u, 1e-9f), 1.f - 1e-9f);
      float noisy = live ? st - logf(-logf(u)) : -INFINITY;
      int ni = live ? lane : 32;
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, noisy, o);
        const int oi = __shfl_xor_sync(0xffffffffu, ni, o);
        if (ov > noisy || (ov == noisy && oi < ni)) { noisy = ov; ni = oi; }
      }
      ch = ni;
    }
    if (live) winp[row + lane] = w;
    const int64_t tok = __shfl_sync(0xffffffffu, c, ch);
    if (lane == 0) drafts[(size_t)b * k + i] = tok;
    prev = tok;
  }
}


// DFlash2 grouped depthwise convolution over block positions (the drafter's DFlashGroupedConv):
//   out[t, c] = sum_{tap <= min(pos(t), taps - 1)} (base[tap, c] + delta[t, tap, c / gs]) h[t - tap, c]
// with pos(t) = t % block (blocks are independent).  One CTA per row, 8 channels per thread,
// fp32 arithmetic, bf16 in and out.
__global__ void __launch_bounds__(128) dflash_conv_kernel(
    const __nv_bfloat16* __restrict__ h, int ldh, const __nv_bfloat16* __restrict__ delta,
    int ldd, const __nv_bfloat16* __restrict__ base, int H, int G, int taps, int block,
    __nv_bfloat16* __restrict__ out, int ldo) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int pos = t % block;
  const int gs = H / G;
  const int nt = min(pos + 1, taps);
  for (int v = threadIdx.x; v < H / 8; v += blockDim.x) {
    const int c = v * 8;
    const int g = c / gs;                   // gs % 8 == 0: the 8 channels share a group
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int tap = 0; tap < nt; ++tap) {
      const float d = __bfloat162float(delta[(size_t)t * ldd + tap * G + g]);
      const uint4 hu = *reinterpret_cast<const uint4*>(h + (size_t)(t - tap) * ldh + c);
      const uint4 bu = *reinterpret_cast<const uint4*>(base + (size_t)tap * H + c);
      const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&hu);
      const __nv_bfloat162* bb = reinterpret_cast<const __nv_bfloat162*>(&bu);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 hf = __bfloat1622float2(hh[i]), bf = __bfloat1622float2(bb[i]);
        acc[2 * i] += (bf.x + d) * hf.x;
        acc[2 * i + 1] += (bf.y + d) * hf.y;
      }
    }
    uint4 o;
    __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int i = 0; i < 4; ++i) oh[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
    *reinterpret_cast<uint4*>(out + (size_t)t * ldo + c) = o;
  }
}
}  // namespace spec

// draft [B,k] int64; t_ids/t_probs [B,k+1,W]; d_ids/d_probs [B,k,Kd] or empty (point mass);
// greedy [B] bool; seq_lens [B] int64; forced [B] int64 or empty; seeds [B] int64.
void rejection_sample_cuda(torch::Tensor draft, torch::Tensor t_ids, torch::Tensor t_probs,
                           torch::Tensor d_ids, torch::Tensor d_probs, torch::Tensor greedy,
                           torch::Tensor seq_lens, torch::Tensor forced, torch::Tensor seeds,
                           int64_t kind, double delta, int64_t fade_start, int64_t fade_end,
                           double cap_r, double escape, double theta, torch::Tensor out,
                           torch::Tensor n_acc) {
  const int B = draft.size(0), k = draft.size(1), W = t_ids.size(2);
  if (B == 0) return;
  TORCH_CHECK(W <= spec::kWin && t_ids.size(1) == k + 1, "rejection: target window <= 64");
  const bool has_d = d_ids.defined() && d_ids.numel();
  const int Kd = has_d ? d_ids.size(2) : 0;
  TORCH_CHECK(!has_d || Kd <= spec::kWin, "rejection: draft window <= 64");
  TORCH_CHECK(t_probs.scalar_type() == at::kFloat && greedy.scalar_type() == at::kBool, "dtypes");
  const at::cuda::CUDAGuard guard(draft.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  spec::Rule rule{(int)kind, (float)delta, (int)fade_start, (int)fade_end, (float)cap_r,
                  (float)escape, (float)theta};
  const int warps = 4;
  C10_CUDA_CHECK(launch_pdl(spec::rejection_kernel, dim3((B + warps - 1) / warps), dim3(32 * warps), 0,
      stream, draft.data_ptr<int64_t>(), k, t_ids.data_ptr<int64_t>(), t_probs.data_ptr<float>(), W,
      has_d ? d_ids.data_ptr<int64_t>() : (const int64_t*)nullptr,
      has_d ? d_probs.data_ptr<float>() : (const float*)nullptr, Kd, greedy.data_ptr<bool>(),
      seq_lens.data_ptr<int64_t>(),
      forced.defined() && forced.numel() ? forced.data_ptr<int64_t>() : (const int64_t*)nullptr,
      seeds.data_ptr<int64_t>(), rule, B, out.data_ptr<int64_t>(), n_acc.data_ptr<int64_t>()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void lookup_draft_cuda(torch::Tensor hist, torch::Tensor rows, torch::Tensor len, int64_t k,
                       int64_t max_ngram, int64_t min_ngram, torch::Tensor out,
                       torch::Tensor n_out) {
  const int B = rows.size(0);
  if (B == 0) return;
  TORCH_CHECK(hist.scalar_type() == at::kInt && len.scalar_type() == at::kInt, "int32 histories");
  const at::cuda::CUDAGuard guard(hist.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  spec::lookup_kernel<<<B, 256, 0, stream>>>(hist.data_ptr<int>(), (int)hist.size(1),
                                             rows.data_ptr<int>(), len.data_ptr<int>(), (int)k,
                                             (int)max_ngram,
                                             (int)min_ngram, out.data_ptr<int>(),
                                             n_out.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace rad

namespace rad {
// unary f32 [B, k, Kc]; cand i64 [B, k, Kc]; anchors i64 [B]; hp f32 [B, k, r];
// pred / succ bf16 [V, r]; temps f32 [B]; seeds i64 [B] -> drafts i64 [B, k], winp f32 [B, k, Kc]
void dflash_walk(torch::Tensor unary, torch::Tensor cand, torch::Tensor anchors, torch::Tensor hp,
                 torch::Tensor pred, torch::Tensor succ, torch::Tensor temps, torch::Tensor seeds,
                 torch::Tensor drafts, torch::Tensor winp, torch::Tensor status) {
  const int B = unary.size(0), k = unary.size(1), Kc = unary.size(2), r = hp.size(2);
  TORCH_CHECK(Kc >= 1 && Kc <= 32, "dflash_walk: 1..32 candidates");
  TORCH_CHECK(unary.scalar_type() == at::kFloat && unary.is_contiguous() &&
                  cand.scalar_type() == at::kLong && cand.is_contiguous() &&
                  cand.numel() == unary.numel() && anchors.scalar_type() == at::kLong &&
                  anchors.numel() >= B && hp.scalar_type() == at::kFloat && hp.is_contiguous() &&
                  hp.size(0) == B && hp.size(1) == k && pred.scalar_type() == at::kBFloat16 &&
                  succ.scalar_type() == at::kBFloat16 && pred.is_contiguous() &&
                  succ.is_contiguous() && pred.size(1) == r && succ.size(1) == r &&
                  pred.size(0) == succ.size(0) && temps.scalar_type() == at::kFloat &&
                  temps.numel() >= B && seeds.scalar_type() == at::kLong && seeds.numel() >= B &&
                  drafts.scalar_type() == at::kLong && drafts.numel() >= (int64_t)B * k &&
                  winp.scalar_type() == at::kFloat && winp.is_contiguous() &&
                  winp.numel() >= unary.numel(), "dflash_walk: args");
  if (B == 0) return;
  const at::cuda::CUDAGuard guard(unary.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  C10_CUDA_CHECK(launch_pdl(spec::walk_kernel, dim3((B + 3) / 4), dim3(128), 0, stream,
                            unary.data_ptr<float>(), cand.data_ptr<int64_t>(),
                            anchors.data_ptr<int64_t>(), hp.data_ptr<float>(),
                            (const __nv_bfloat16*)pred.data_ptr(),
                            (const __nv_bfloat16*)succ.data_ptr(), temps.data_ptr<float>(),
                            seeds.data_ptr<int64_t>(), B, k, Kc, r, (int64_t)pred.size(0),
                            drafts.data_ptr<int64_t>(), winp.data_ptr<float>(),
                            status.data_ptr<int>()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
// h [T, H] bf16 (rows 16-byte aligned); delta: bf16 view [T, taps, G] with row stride ldd and
// unit group stride; base bf16 [taps, H]; out [T, H] bf16.
void dflash_conv(torch::Tensor h, torch::Tensor delta, torch::Tensor base, int64_t G,
                 int64_t block, torch::Tensor out) {
  const int T = h.size(0), H = h.size(1), taps = base.size(0);
  TORCH_CHECK(h.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16 &&
                  base.scalar_type() == at::kBFloat16 && delta.scalar_type() == at::kBFloat16,
              "dflash_conv: bf16 tensors");
  TORCH_CHECK(h.stride(1) == 1 && h.stride(0) % 8 == 0 && out.stride(1) == 1 &&
                  out.stride(0) % 8 == 0 && base.is_contiguous() && base.size(1) == H,
              "dflash_conv: row layouts");
  TORCH_CHECK(H % 8 == 0 && G >= 1 && H % G == 0 && (H / G) % 8 == 0, "dflash_conv: groups");
  TORCH_CHECK(delta.dim() == 3 && delta.size(0) == T && delta.size(1) == taps &&
                  delta.size(2) == G && delta.stride(2) == 1 && delta.stride(1) == G,
              "dflash_conv: delta [T, taps, G]");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(h.data_ptr()) % 16) == 0 &&
                  (reinterpret_cast<uintptr_t>(out.data_ptr()) % 16) == 0 &&
                  (reinterpret_cast<uintptr_t>(base.data_ptr()) % 16) == 0, "dflash_conv: alignment");
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(h.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  C10_CUDA_CHECK(launch_pdl(spec::dflash_conv_kernel, dim3(T), dim3(128), 0, stream,
                            (const __nv_bfloat16*)h.data_ptr(), (int)h.stride(0),
                            (const __nv_bfloat16*)delta.data_ptr(), (int)delta.stride(0),
                            (const __nv_bfloat16*)base.data_ptr(), H, (int)G, taps, (int)block,
                            (__nv_bfloat16*)out.data_ptr(), (int)out.stride(0)));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
}  // namespace rad
