// Gated delta net (GDN) linear-attention kernels.
//
// Reference behaviour: libr4d gdn_conv_prep / gdn_conv_update (radiance_gdn.py:444,466), the
// recurrent update gdn_recurrent_update_* and the fused decode kernel
// (sly/gdn/radiance_gdn_decode.hip:140), with the fp64 oracle sly/gdn/chunk_scan_ref.py:48-110:
//   S <- e^g S;  S <- S + beta (v - S k) k^T;  o = scale * S q      (S is [dv, dk] per v-head)
//   g = -exp(A_log) * softplus(a + dt_bias),  beta = sigmoid(b)
//
// Kernels here:
//  * gdn_conv       : varlen depthwise causal conv (width W) over [q|k|v] channels + SiLU, with the
//                     per-sequence conv state as left context, q/k L2-normalised per head in the
//                     same pass.  Serves prefill chunks and decode tokens alike.
//  * gdn_conv_state : writes each sequence's new conv state (separate launch: the conv kernel
//                     still reads the old state for the first W-1 tokens of every sequence).
//  * gdn_recurrent  : varlen token-serial delta rule with the state held in registers, one CTA per
//                     (sequence, v-head, 32-row slice of dv).  Used for decode / verify rows and,
//                     until the chunked scan lands, for prefill rows as well.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdlib>

#include "common.cuh"

namespace rad {
namespace gdn {

// ------------------------------------------------------------------------------------------------
// conv: grid (T, ceil(num_chunks / 8)), block 256 (8 warps); warp handles one D-channel chunk
// (D = head dim, q/k/v heads all D wide) of one token.
// ------------------------------------------------------------------------------------------------
template <int D, int W>
__global__ void __launch_bounds__(256) conv_kernel(
    const __nv_bfloat16* __restrict__ x, int ldx, const __nv_bfloat16* __restrict__ w,
    const __nv_bfloat16* __restrict__ conv_state, const int* __restrict__ qsl,
    const int* __restrict__ slots, const int* __restrict__ has_init, const int* __restrict__ tok_seq,
    int C, int qk_dim, __nv_bfloat16* __restrict__ y, int ldy, float eps, int update_state) {
  pdl_wait();     // inputs come from the preceding kernel
  pdl_trigger();
  constexpr int PER = D / 32;           // channels per lane
  const int t = blockIdx.x;
  const int chunk = blockIdx.y * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (chunk * D >= C) return;
  const int b = tok_seq[t];
  const int s0 = qsl[b];
  const int i = t - s0;                 // position within this step's tokens
  const int slot = slots[b];
  const bool init = has_init[b] != 0;
  float acc[PER];
  float xin[W][PER];
#pragma unroll
  for (int p = 0; p < PER; ++p) acc[p] = 0.f;
#pragma unroll
  for (int j = 0; j < W; ++j) {
    // input index i + j - (W-1) relative to the first token of the step
    const int src = i + j - (W - 1);
#pragma unroll
    for (int p = 0; p < PER; ++p) {
      const int c = chunk * D + lane * PER + p;
      float xv;
      if (src >= 0) {
        xv = __bfloat162float(x[(size_t)(s0 + src) * ldx + c]);
      } else {
        // state holds the previous W-1 inputs, oldest first: state[W-1+src]
        xv = init ? __bfloat162float(conv_state[((size_t)slot * C + c) * (W - 1) + (W - 1 + src)]) : 0.f;
      }
      xin[j][p] = xv;
      acc[p] += xv * __bfloat162float(w[(size_t)c * W + j]);
    }
  }
  if (update_state) {
    // decode (one token per sequence): this warp is the only reader of these state entries, so
    // it shifts them in place (the separate state-update launch is skipped)
#pragma unroll
    for (int p = 0; p < PER; ++p) {
      const int c = chunk * D + lane * PER + p;
      __nv_bfloat16* st = const_cast<__nv_bfloat16*>(conv_state) + ((size_t)slot * C + c) * (W - 1);
#pragma unroll
      for (int j = 0; j < W - 1; ++j) st[j] = __float2bfloat16_rn(xin[j + 1][p]);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int p = 0; p < PER; ++p) {
    acc[p] = acc[p] / (1.f + __expf(-acc[p]));
    ss += acc[p] * acc[p];
  }
  if (chunk * D < qk_dim) {
    ss = warp_sum(ss);
    const float r = rsqrtf(ss + eps);
#pragma unroll
    for (int p = 0; p < PER; ++p) acc[p] *= r;
  }
#pragma unroll
  for (int p = 0; p < PER; ++p)
    y[(size_t)t * ldy + chunk * D + lane * PER + p] = __float2bfloat16_rn(acc[p]);
}

// Prefill conv, token-tiled: a warp owns one D-channel chunk of TT consecutive tokens; lane l
// keeps 4 channels.  The TT + W - 1 input rows the tile reads are loaded once (8-byte vectors)
// and slide through the W taps, instead of every output re-reading its W inputs; taps are fetched
// before the dependency wait.  Rows of another sequence (varlen batches) come from the sequence's
// saved conv state, as in conv_kernel.
template <int D, int W, int TT>
__global__ void __launch_bounds__(256) conv_tile_kernel(
    const __nv_bfloat16* __restrict__ x, int ldx, const __nv_bfloat16* __restrict__ w,
    const __nv_bfloat16* __restrict__ conv_state, const int* __restrict__ qsl,
    const int* __restrict__ slots, const int* __restrict__ has_init, const int* __restrict__ tok_seq,
    int T, int C, int qk_dim, __nv_bfloat16* __restrict__ y, int ldy, float eps) {
  static_assert(D == 128 && W == 4, "4 channels per lane, 4 taps");
  const int chunk = blockIdx.y * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int c0 = chunk * D + lane * 4;
  const bool live = chunk * D < C;
  float wt[4][W];                       // [channel][tap]
  if (live) {
    const uint4 wa = *reinterpret_cast<const uint4*>(w + (size_t)c0 * W);
    const uint4 wb = *reinterpret_cast<const uint4*>(w + (size_t)c0 * W + 8);
    const __nv_bfloat162* ha = reinterpret_cast<const __nv_bfloat162*>(&wa);
    const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&wb);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 fa = __bfloat1622float2(ha[e]), fb = __bfloat1622float2(hb[e]);
      wt[e / 2][(e % 2) * 2] = fa.x;
      wt[e / 2][(e % 2) * 2 + 1] = fa.y;
      wt[2 + e / 2][(e % 2) * 2] = fb.x;
      wt[2 + e / 2][(e % 2) * 2 + 1] = fb.y;
    }
  }
  pdl_wait();     // the in_proj output comes from the preceding kernel
  pdl_trigger();
  if (!live) return;
  const int t0 = blockIdx.x * TT;
  // rows t0 - (W - 1) .. t0 + TT - 1 (clamped; a clamped row is never used as a same-sequence input)
  float xr[TT + W - 1][4];
#pragma unroll
  for (int j = 0; j < TT + W - 1; ++j) {
    const int r = min(max(t0 - (W - 1) + j, 0), T - 1);
    const uint2 u = *reinterpret_cast<const uint2*>(x + (size_t)r * ldx + c0);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    const float2 a = __bfloat1622float2(h[0]), b2 = __bfloat1622float2(h[1]);
    xr[j][0] = a.x; xr[j][1] = a.y; xr[j][2] = b2.x; xr[j][3] = b2.y;
  }
  const bool qk = chunk * D < qk_dim;
#pragma unroll
  for (int k = 0; k < TT; ++k) {
    const int t = t0 + k;
    if (t >= T) break;                  // uniform across the warp
    const int b = tok_seq[t];
    const int i = t - qsl[b];           // position within the sequence's tokens of this step
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < W; ++j) {
      const int src = i + j - (W - 1);
      float v[4];
      if (src >= 0) {
#pragma unroll
        for (int p = 0; p < 4; ++p) v[p] = xr[k + j][p];
      } else {
        const bool init = has_init[b] != 0;
        const int slot = slots[b];
#pragma unroll
        for (int p = 0; p < 4; ++p)
          v[p] = init ? __bfloat162float(conv_state[((size_t)slot * C + c0 + p) * (W - 1) + (W - 1 + src)])
                      : 0.f;
      }
#pragma unroll
      for (int p = 0; p < 4; ++p) acc[p] += v[p] * wt[p][j];
    }
    float ss = 0.f;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      acc[p] = acc[p] / (1.f + __expf(-acc[p]));
      ss += acc[p] * acc[p];
    }
    if (qk) {
      ss = warp_sum(ss);
      const float r = rsqrtf(ss + eps);
#pragma unroll
      for (int p = 0; p < 4; ++p) acc[p] *= r;
    }
    uint2 o;
    __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
    oh[0] = __floats2bfloat162_rn(acc[0], acc[1]);
    oh[1] = __floats2bfloat162_rn(acc[2], acc[3]);
    *reinterpret_cast<uint2*>(y + (size_t)t * ldy + c0) = o;
  }
}

// new state for each sequence = the last W-1 inputs of concat(old_state, x_seq[:n_commit])
template <int W>
__global__ void conv_state_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                                  __nv_bfloat16* __restrict__ conv_state,
                                  const int* __restrict__ qsl, const int* __restrict__ slots,
                                  const int* __restrict__ has_init,
                                  const int* __restrict__ commit_len, int C) {
  pdl_wait();     // inputs come from the preceding kernel
  pdl_trigger();
  const int b = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int s0 = qsl[b];
  const int L = commit_len ? commit_len[b] : (qsl[b + 1] - s0);
  if (L < 0) return;                    // row not part of this commit pass
  const int slot = slots[b];
  const bool init = has_init[b] != 0;
  __nv_bfloat16* st = conv_state + ((size_t)slot * C + c) * (W - 1);
  float old[W - 1];
#pragma unroll
  for (int j = 0; j < W - 1; ++j) old[j] = init ? __bfloat162float(st[j]) : 0.f;
  float nw[W - 1];
#pragma unroll
  for (int j = 0; j < W - 1; ++j) {
    // element j of the new state is input index L - (W-1) + j (negative -> old state)
    const int src = L - (W - 1) + j;
    nw[j] = src >= 0 ? __bfloat162float(x[(size_t)(s0 + src) * ldx + c]) : old[W - 1 + src];
  }
#pragma unroll
  for (int j = 0; j < W - 1; ++j) st[j] = __float2bfloat16_rn(nw[j]);
}

// ------------------------------------------------------------------------------------------------
// recurrent delta rule.  grid (B, Hv, DV / 32), block 128: warp w owns rows [8w, 8w+8) of the
// 32-row slice, lane owns dk columns [lane*DK/32, ...).
// ------------------------------------------------------------------------------------------------
template <int DK, typename ST>
__global__ void __launch_bounds__(128) recurrent_kernel(
    const __nv_bfloat16* __restrict__ y, int ldy,        // conv output [T, C]: q | k | v
    const __nv_bfloat16* __restrict__ ba, int ldba,      // [T, ...]: b at col 0.., a at col Hv..
    const float* __restrict__ A_log, const float* __restrict__ dt_bias,
    ST* __restrict__ state,                              // [S, Hv, DV, DK]
    const int* __restrict__ qsl, const int* __restrict__ slots, const int* __restrict__ has_init,
    const int* __restrict__ commit_len,                  // optional: rows to apply to the stored state
    int Hk, int Hv, int DV, float scale, __nv_bfloat16* __restrict__ out, int ldo,
    int write_out) {
  pdl_wait();     // inputs come from the preceding kernel
  pdl_trigger();
  constexpr int PL = DK / 32;          // dk columns per lane
  constexpr int RW = 8;                // rows per warp
  const int b = blockIdx.x;
  const int h = blockIdx.y;
  const int r0 = blockIdx.z * 32 + (threadIdx.x / 32) * RW;
  const int lane = threadIdx.x % 32;
  const int s0 = qsl[b];
  const int L = qsl[b + 1] - s0;
  const int Lc = commit_len ? commit_len[b] : L;
  if (Lc < 0) return;                   // row not part of this commit pass
  const int Lrun = write_out ? L : min(L, Lc);
  const int slot = slots[b];
  const int hk = h / (Hv / Hk);
  const int key_dim = Hk * DK;
  const float negA = -__expf(A_log[h]);
  const float dtb = dt_bias[h];

  float S[RW][PL];
  ST* sp = state + (((size_t)slot * Hv + h) * DV + r0) * DK + lane * PL;
  if (has_init[b]) {
#pragma unroll
    for (int r = 0; r < RW; ++r)
#pragma unroll
      for (int p = 0; p < PL; ++p) S[r][p] = to_f(sp[(size_t)r * DK + p]);
  } else {
#pragma unroll
    for (int r = 0; r < RW; ++r)
#pragma unroll
      for (int p = 0; p < PL; ++p) S[r][p] = 0.f;
  }

  for (int i = 0; i < Lrun; ++i) {
    const size_t t = s0 + i;
    const __nv_bfloat16* yt = y + t * ldy;
    float q[PL], k[PL], v[RW];
#pragma unroll
    for (int p = 0; p < PL; ++p) {
      q[p] = __bfloat162float(yt[hk * DK + lane * PL + p]);
      k[p] = __bfloat162float(yt[key_dim + hk * DK + lane * PL + p]);
    }
#pragma unroll
    for (int r = 0; r < RW; ++r) v[r] = __bfloat162float(yt[2 * key_dim + h * DV + r0 + r]);
    const float bb = __bfloat162float(ba[t * ldba + h]);
    const float aa = __bfloat162float(ba[t * ldba + Hv + h]);
    const float xsp = aa + dtb;
    const float sp_ = xsp > 20.f ? xsp : log1pf(__expf(xsp));
    const float decay = __expf(negA * sp_);
    const float beta = 1.f / (1.f + __expf(-bb));
    float kv[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
      float acc = 0.f;
#pragma unroll
      for (int p = 0; p < PL; ++p) {
        S[r][p] *= decay;
        acc += S[r][p] * k[p];
      }
      kv[r] = acc;
    }
#pragma unroll
    for (int r = 0; r < RW; ++r) kv[r] = warp_sum(kv[r]);
    float o[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
      const float d = beta * (v[r] - kv[r]);
      float acc = 0.f;
#pragma unroll
      for (int p = 0; p < PL; ++p) {
        S[r][p] += d * k[p];
        acc += S[r][p] * q[p];
      }
      o[r] = acc;
    }
#pragma unroll
    for (int r = 0; r < RW; ++r) o[r] = warp_sum(o[r]);
    if (write_out && lane < RW) {
      float ov = 0.f;
#pragma unroll
      for (int r = 0; r < RW; ++r)
        if (r == lane) ov = o[r];
      out[t * ldo + h * DV + r0 + lane] = __float2bfloat16_rn(ov * scale);
    }
    if (i + 1 == Lc) {
#pragma unroll
      for (int r = 0; r < RW; ++r)
#pragma unroll
        for (int p = 0; p < PL; ++p) sp[(size_t)r * DK + p] = from_f<ST>(S[r][p]);
    }
  }
}


// ------------------------------------------------------------------------------------------------
// fused decode step (one token per sequence): conv update + SiLU + q/k L2 norm + gates + delta
// rule in one launch (the reference's gdn_fused_update / radiance_gdn_decode.hip:140 step).
// grid (B, Hv), 256 threads; the rep = Hv / Hk value heads that share one q/k head form a thread
// block cluster: each computes the shared q/k conv itself, and after a cluster barrier (every
// CTA has read the old q/k conv state) only cluster rank 0 writes the shifted q/k state.  A
// thread pair owns one row of the [dv, dk] state (64 columns each): one shuffle per reduction.
// ------------------------------------------------------------------------------------------------
// The out_proj producer fused into the decode step (FQ): the CTA of head h applies the gated
// RMSNorm to its own 128 outputs -- n = bf16(bf16(o * rsqrt(mean_head(o^2) + eps) * w) * silu(z))
// with o = bf16(scale * S q), the numerics of gdn_norm_quant -- writes them with the head's amax,
// and the last head CTA of the row (self-resetting per-row counter) quantises the whole row to
// e4m3 with its per-token scale.
struct GdnQuantArgs {
  int z_off;                       // column of z in the in_proj output row
  const __nv_bfloat16* norm_w;     // [D]
  float norm_eps;
  __nv_bfloat16* nout;             // [B, Hv * D] normed row (bf16 scratch)
  float* head_amax;                // [B, Hv]
  unsigned* row_cnt;               // [B] arrival counters (zero, self-resetting)
  uint8_t* q;                      // [B, Hv * D] e4m3
  int ldq;
  float* q_scale;                  // [B]
};

template <int D, typename ST, int NS, bool FQ = false>
__global__ void __launch_bounds__(2 * D) decode_fused_kernel(
    const __nv_bfloat16* __restrict__ x, int ldx,        // in_proj output [B, *]: q|k|v|z|b|a
    const __nv_bfloat16* __restrict__ conv_w,            // [C, 4]
    __nv_bfloat16* __restrict__ conv_state,              // [S, C, 3]
    int ba_off,                                          // column of b (a at ba_off + Hv)
    const float* __restrict__ A_log, const float* __restrict__ dt_bias,
    ST* __restrict__ state,                              // [S, Hv, D, D]
    const int* __restrict__ slots, const int* __restrict__ has_init, int Hk, int Hv, int C,
    float scale, float eps, __nv_bfloat16* __restrict__ out, int ldo, const GdnQuantArgs fq) {
  constexpr int W = 4;
  // model constants (conv taps of this thread's q / k / v channels, the head's gate parameters)
  // are fetched before the dependency wait, overlapping the predecessor's tail
  float cwq[W], cwk[W], cwv[W];
  {
    const int hk0 = blockIdx.y / (Hv / Hk);
    const int tt = threadIdx.x;
    if (tt < D) {
      const int cq = hk0 * D + tt, ck = Hk * D + hk0 * D + tt, cv = 2 * Hk * D + blockIdx.y * D + tt;
#pragma unroll
      for (int j = 0; j < W; ++j) {
        cwq[j] = __bfloat162float(conv_w[(size_t)cq * W + j]);
        cwk[j] = __bfloat162float(conv_w[(size_t)ck * W + j]);
        cwv[j] = __bfloat162float(conv_w[(size_t)cv * W + j]);
      }
    }
  }
  const float a_log = A_log[blockIdx.y], dtb = dt_bias[blockIdx.y];
  float nw = 0.f;
  if constexpr (FQ) {
    static_assert(NS == 1, "the fused norm needs the head's outputs in one CTA");
    if (threadIdx.x < D) nw = __bfloat162float(fq.norm_w[threadIdx.x]);
  }
  constexpr int TPR = 2 * NS;           // threads per state row
  constexpr int RPC = D / NS;           // state rows of this CTA (blockIdx.z picks which)
  constexpr int HC = D / TPR;           // state columns per thread
  static_assert(RPC * TPR == 2 * D, "2 * D threads cover the CTA's rows");
  __shared__ float sq[D], sk[D], sv[D], sred[2][D / 32];
  const int b = blockIdx.x, h = blockIdx.y, z = blockIdx.z;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int rep = Hv / Hk, hk = h / rep;
  const int key_dim = Hk * D;
  const int slot = slots[b];
  const bool init = has_init[b] != 0;
  const __nv_bfloat16* xr = x + (size_t)b * ldx;
  // ---- this thread's slice of its state row, loaded first so the load overlaps the conv ----
  const int r = z * RPC + t / TPR, c0 = (t % TPR) * HC;
  ST* srow = state + (((size_t)slot * Hv + h) * D + r) * D + c0;
  float S[HC];
  if (init) {
    if constexpr (sizeof(ST) == 4) {
#pragma unroll
      for (int c = 0; c < HC; c += 4) {
        const float4 f = *reinterpret_cast<const float4*>(srow + c);
        S[c] = f.x; S[c + 1] = f.y; S[c + 2] = f.z; S[c + 3] = f.w;
      }
    } else {
#pragma unroll
      for (int c = 0; c < HC; c += 8) {
        const uint4 u = *reinterpret_cast<const uint4*>(srow + c);
        const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(hh[e]);
          S[c + 2 * e] = f.x;
          S[c + 2 * e + 1] = f.y;
        }
      }
    }
  } else {
#pragma unroll
    for (int c = 0; c < HC; ++c) S[c] = 0.f;
  }
  // ---- conv (threads 0..D-1, one channel of q, k and v each) + SiLU + q/k L2 norm ----
  float in_q[W], in_k[W], in_v[W];
  __nv_bfloat16 *stq = nullptr, *stk = nullptr, *stv = nullptr;
  const int cq = hk * D + t, ck = key_dim + hk * D + t, cv = 2 * key_dim + h * D + t;
  if (t < D) {
    stq = conv_state + ((size_t)slot * C + cq) * (W - 1);
    stk = conv_state + ((size_t)slot * C + ck) * (W - 1);
    stv = conv_state + ((size_t)slot * C + cv) * (W - 1);
#pragma unroll
    for (int j = 0; j < W - 1; ++j) {
      in_q[j] = init ? __bfloat162float(stq[j]) : 0.f;
      in_k[j] = init ? __bfloat162float(stk[j]) : 0.f;
      in_v[j] = init ? __bfloat162float(stv[j]) : 0.f;
    }
  }
  // The recurrent and conv states (read above) were last written by this layer's kernel one
  // step earlier, and the slot tables come with the step's metadata: only the in_proj row below
  // depends on the kernel before this one, so the state loads overlap that kernel's tail.
  pdl_wait();
  pdl_trigger();
  if (t < D) {
    in_q[W - 1] = __bfloat162float(xr[cq]);
    in_k[W - 1] = __bfloat162float(xr[ck]);
    in_v[W - 1] = __bfloat162float(xr[cv]);
    float aq = 0.f, ak = 0.f, av = 0.f;
#pragma unroll
    for (int j = 0; j < W; ++j) {
      aq += in_q[j] * cwq[j];
      ak += in_k[j] * cwk[j];
      av += in_v[j] * cwv[j];
    }
    aq = aq / (1.f + __expf(-aq));
    ak = ak / (1.f + __expf(-ak));
    av = av / (1.f + __expf(-av));
    const float s2q = warp_sum(aq * aq), s2k = warp_sum(ak * ak);
    if (lane == 0) { sred[0][warp] = s2q; sred[1][warp] = s2k; }
    sq[t] = aq;
    sk[t] = ak;
    sv[t] = bf16_round(av);             // the conv kernel's bf16 output rounding
  }
  __syncthreads();
  if (t < D) {
    float s2q = 0.f, s2k = 0.f;
#pragma unroll
    for (int w = 0; w < D / 32; ++w) { s2q += sred[0][w]; s2k += sred[1][w]; }
    sq[t] = bf16_round(sq[t] * rsqrtf(s2q + eps));
    sk[t] = bf16_round(sk[t] * rsqrtf(s2k + eps));
    // shift the conv state: v channel t belongs to the CTA that owns state row t
    if (t / RPC == z) {
#pragma unroll
      for (int j = 0; j < W - 1; ++j) stv[j] = __float2bfloat16_rn(in_v[j + 1]);
    }
  }
  // q/k state: cluster rank 0, after every CTA of the cluster has read the old q/k state
  cluster_sync();
  if (t < D && z == 0 && cluster_ctarank() == 0) {
#pragma unroll
    for (int j = 0; j < W - 1; ++j) {
      stq[j] = __float2bfloat16_rn(in_q[j + 1]);
      stk[j] = __float2bfloat16_rn(in_k[j + 1]);
    }
  }
  // ---- gates ----
  const float bb = __bfloat162float(xr[ba_off + h]);
  const float aa = __bfloat162float(xr[ba_off + Hv + h]);
  const float xs = aa + dtb;
  const float sp = xs > 20.f ? xs : log1pf(__expf(xs));
  const float decay = __expf(-__expf(a_log) * sp);
  const float beta = 1.f / (1.f + __expf(-bb));
  // ---- delta rule: TPR consecutive threads own row r of S, HC columns each ----
  float kv = 0.f;
#pragma unroll
  for (int c = 0; c < HC; ++c) {
    S[c] *= decay;
    kv += S[c] * sk[c0 + c];
  }
#pragma unroll
  for (int o = 1; o < TPR; o <<= 1) kv += __shfl_xor_sync(0xffffffffu, kv, o);
  const float dlt = beta * (sv[r] - kv);
  float o = 0.f;
#pragma unroll
  for (int c = 0; c < HC; ++c) {
    S[c] += dlt * sk[c0 + c];
    o += S[c] * sq[c0 + c];
  }
#pragma unroll
  for (int m = 1; m < TPR; m <<= 1) o += __shfl_xor_sync(0xffffffffu, o, m);
  if constexpr (!FQ) {
    if (t % TPR == 0) out[(size_t)b * ldo + h * D + r] = __float2bfloat16_rn(o * scale);
  } else {
    if (t % TPR == 0) sv[r] = bf16_round(o * scale);      // v is consumed: reuse its buffer
  }
  if constexpr (sizeof(ST) == 4) {
#pragma unroll
    for (int c = 0; c < HC; c += 4)
      *reinterpret_cast<float4*>(srow + c) = make_float4(S[c], S[c + 1], S[c + 2], S[c + 3]);
  } else {
#pragma unroll
    for (int c = 0; c < HC; c += 8) {
      uint4 u;
      __nv_bfloat162* hh = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) hh[e] = __floats2bfloat162_rn(S[c + 2 * e], S[c + 2 * e + 1]);
      *reinterpret_cast<uint4*>(srow + c) = u;
    }
  }
  if constexpr (FQ) {
    __shared__ bool s_last;
    __syncthreads();
    // gated RMSNorm of the head (threads 0..D-1 own one output each)
    float n = 0.f;
    if (t < D) {
      const float ov = sv[t];
      const float ss = warp_sum(ov * ov);
      if (lane == 0) sred[0][warp] = ss;
    }
    __syncthreads();
    if (t < D) {
      float ss = 0.f;
#pragma unroll
      for (int w = 0; w < D / 32; ++w) ss += sred[0][w];
      const float rs = rsqrtf(ss / (float)D + fq.norm_eps);
      const float zz = __bfloat162float(xr[fq.z_off + h * D + t]);
      const float nn = bf16_round(sv[t] * rs * nw);
      n = bf16_round(nn * (zz / (1.f + __expf(-zz))));
      fq.nout[(size_t)b * Hv * D + h * D + t] = __float2bfloat16_rn(n);
      const float am = warp_max(fabsf(n));
      if (lane == 0) sred[1][warp] = am;
    }
    __syncthreads();
    if (t == 0) {
      float am = 0.f;
#pragma unroll
      for (int w = 0; w < D / 32; ++w) am = fmaxf(am, sred[1][w]);
      fq.head_amax[(size_t)b * Hv + h] = am;
      __threadfence();
      s_last = atomicAdd(&fq.row_cnt[b], 1u) == (unsigned)(Hv - 1);
      if (s_last) fq.row_cnt[b] = 0u;
    }
    __syncthreads();
    if (s_last) {   // every head of row b is normed: quantise the row
      __threadfence();
      float am = 0.f;
      for (int i = lane; i < Hv; i += 32) am = fmaxf(am, __ldcg(fq.head_amax + (size_t)b * Hv + i));
      am = warp_max(am);
      const float qs = fmaxf(am / 448.f, 1.f / (448.f * 512.f));
      const float inv = 1.f / qs;
      const int H = Hv * D;
      for (int v = t; v < H / 8; v += 2 * D) {
        const uint4 u = __ldcg(reinterpret_cast<const uint4*>(fq.nout + (size_t)b * H + v * 8));
        const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&u);
        uint2 qq;
        uint16_t* q16 = reinterpret_cast<uint16_t*>(&qq);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(hh[e]);
          q16[e] = f32x2_to_e4m3x2(f.x * inv, f.y * inv);
        }
        *reinterpret_cast<uint2*>(fq.q + (size_t)b * fq.ldq + v * 8) = qq;
      }
      if (t == 0) fq.q_scale[b] = qs;
    }
  }
}

}  // namespace gdn

static inline const int* iptr(const torch::Tensor& t) {
  return t.defined() && t.numel() ? t.data_ptr<int>() : nullptr;
}

// x: [T, >=C] bf16 (qkv part of in_proj output), w [C, W], conv_state [S, C, W-1] bf16,
// qsl [B+1], slots [B], has_init [B], tok_seq [T] (sequence index of each token), y [T, C] out
void gdn_conv(torch::Tensor x, torch::Tensor w, torch::Tensor conv_state, torch::Tensor qsl,
              torch::Tensor slots, torch::Tensor has_init, torch::Tensor tok_seq, int64_t qk_dim,
              int64_t head_dim, torch::Tensor y, double eps, bool update_state) {
  const int T = x.size(0);
  const int C = w.size(0), W = w.size(1);
  if (T == 0) return;
  TORCH_CHECK(W == 4, "gdn_conv: conv width 4 supported");
  TORCH_CHECK(C % head_dim == 0 && qk_dim % head_dim == 0, "gdn_conv: dims");
  const at::cuda::CUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int chunks = C / head_dim;
  if (!update_state && head_dim == 128 && T > 1 && (x.stride(0) % 4) == 0 &&
      (y.stride(0) % 4) == 0 && (reinterpret_cast<uintptr_t>(x.data_ptr()) % 8) == 0 &&
      (reinterpret_cast<uintptr_t>(y.data_ptr()) % 8) == 0 &&
      (reinterpret_cast<uintptr_t>(w.data_ptr()) % 16) == 0) {
    // prefill: token tiles of 8 (each input row loaded once per tile)
    constexpr int TT = 8;
    C10_CUDA_CHECK(launch_pdl((gdn::conv_tile_kernel<128, 4, TT>), dim3((T + TT - 1) / TT, (chunks + 7) / 8),
        dim3(256), 0, stream, (const __nv_bfloat16*)x.data_ptr(), (int)x.stride(0),
        (const __nv_bfloat16*)w.data_ptr(), (const __nv_bfloat16*)conv_state.data_ptr(),
        qsl.data_ptr<int>(), slots.data_ptr<int>(), has_init.data_ptr<int>(),
        tok_seq.data_ptr<int>(), T, C, (int)qk_dim, (__nv_bfloat16*)y.data_ptr(), (int)y.stride(0),
        (float)eps));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  dim3 grid(T, (chunks + 7) / 8);
  auto run = [&](auto dtag) {
    constexpr int D = decltype(dtag)::value;
C10_CUDA_CHECK(launch_pdl((gdn::conv_kernel<D, 4>), dim3(grid), dim3(256), 0, stream, 
        (const __nv_bfloat16*)x.data_ptr(), x.stride(0), (const __nv_bfloat16*)w.data_ptr(),
        (const __nv_bfloat16*)conv_state.data_ptr(), qsl.data_ptr<int>(), slots.data_ptr<int>(),
        has_init.data_ptr<int>(), tok_seq.data_ptr<int>(), C, qk_dim,
        (__nv_bfloat16*)y.data_ptr(), y.stride(0), (float)eps, update_state ? 1 : 0));
  };
  if (head_dim == 128) run(std::integral_constant<int, 128>{});
  else if (head_dim == 64) run(std::integral_constant<int, 64>{});
  else TORCH_CHECK(false, "gdn_conv: head_dim 64 or 128");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gdn_conv_state_update(torch::Tensor x, torch::Tensor conv_state, torch::Tensor qsl,
                           torch::Tensor slots, torch::Tensor has_init, torch::Tensor commit_len) {
  const int B = slots.size(0);
  const int C = conv_state.size(1), W = conv_state.size(2) + 1;
  if (B == 0) return;
  TORCH_CHECK(W == 4, "gdn_conv_state_update: width 4");
  const at::cuda::CUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  dim3 grid((C + 255) / 256, B);
C10_CUDA_CHECK(launch_pdl((gdn::conv_state_kernel<4>), dim3(grid), dim3(256), 0, stream, 
      (const __nv_bfloat16*)x.data_ptr(), x.stride(0), (__nv_bfloat16*)conv_state.data_ptr(),
      qsl.data_ptr<int>(), slots.data_ptr<int>(), has_init.data_ptr<int>(), iptr(commit_len), C));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gdn_recurrent(torch::Tensor y, torch::Tensor ba, torch::Tensor A_log, torch::Tensor dt_bias,
                   torch::Tensor state, torch::Tensor qsl, torch::Tensor slots,
                   torch::Tensor has_init, torch::Tensor commit_len, int64_t Hk, double scale,
                   torch::Tensor out, bool write_out) {
  const int B = slots.size(0);
  if (B == 0) return;
  const int Hv = state.size(1), DV = state.size(2), DK = state.size(3);
  TORCH_CHECK(DV % 32 == 0, "gdn_recurrent: dv % 32");
  TORCH_CHECK(A_log.scalar_type() == at::kFloat && dt_bias.scalar_type() == at::kFloat, "fp32 gates");
  const at::cuda::CUDAGuard guard(y.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  dim3 grid(B, Hv, DV / 32);
  auto run = [&](auto dtag, auto stag) {
    constexpr int DKc = decltype(dtag)::value;
    using ST = typename decltype(stag)::type;
C10_CUDA_CHECK(launch_pdl((gdn::recurrent_kernel<DKc, ST>), dim3(grid), dim3(128), 0, stream, 
        (const __nv_bfloat16*)y.data_ptr(), y.stride(0), (const __nv_bfloat16*)ba.data_ptr(),
        ba.stride(0), A_log.data_ptr<float>(), dt_bias.data_ptr<float>(), (ST*)state.data_ptr(),
        qsl.data_ptr<int>(), slots.data_ptr<int>(), has_init.data_ptr<int>(), iptr(commit_len),
        Hk, Hv, DV, (float)scale, out.defined() && out.numel() ? (__nv_bfloat16*)out.data_ptr() : nullptr,
        out.defined() && out.numel() ? out.stride(0) : 0, write_out ? 1 : 0));
  };
  struct F32 { using type = float; };
  struct BF16 { using type = __nv_bfloat16; };
  const bool f32 = state.scalar_type() == at::kFloat;
  if (DK == 128) {
    if (f32) run(std::integral_constant<int, 128>{}, F32{});
    else run(std::integral_constant<int, 128>{}, BF16{});
  } else if (DK == 64) {
    if (f32) run(std::integral_constant<int, 64>{}, F32{});
    else run(std::integral_constant<int, 64>{}, BF16{});
  } else {
    TORCH_CHECK(false, "gdn_recurrent: dk 64 or 128");
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}


// One-token-per-sequence GDN step fused into one launch (see decode_fused_kernel).  x = in_proj
// output rows, ba_off = column of the b gates; out = [B, Hv * dv] bf16.
// With q defined (fused norm + quant): z_off = column of z in x, norm_w [128] (gated RMSNorm
// weight), norm_eps, nout bf16 [B, Hv * 128] scratch, ws int32 workspace (>= 4096 + B * Hv
// elements: per-row counters at [0, 4096), zero, self-resetting; then the head amax slots),
// q e4m3 [B, Hv * 128], q_scale [B].
void gdn_decode_fused(torch::Tensor x, int64_t ba_off, torch::Tensor conv_w,
                      torch::Tensor conv_state, torch::Tensor A_log, torch::Tensor dt_bias,
                      torch::Tensor state, torch::Tensor slots, torch::Tensor has_init, int64_t Hk,
                      double scale, double eps, torch::Tensor out, int64_t split, int64_t z_off,
                      torch::Tensor norm_w, double norm_eps, torch::Tensor nout, torch::Tensor ws,
                      torch::Tensor q, torch::Tensor q_scale) {
  const int B = slots.size(0);
  if (B == 0) return;
  const int Hv = state.size(1), DV = state.size(2), DK = state.size(3);
  const int C = conv_w.size(0);
  TORCH_CHECK(DV == 128 && DK == 128, "gdn_decode_fused: dk = dv = 128");
  TORCH_CHECK(conv_w.size(1) == 4 && conv_state.size(2) == 3, "gdn_decode_fused: conv width 4");
  TORCH_CHECK(Hv % Hk == 0 && Hv / Hk <= 8, "gdn_decode_fused: value heads per key head <= 8");
  TORCH_CHECK(x.size(0) >= B && x.stride(1) == 1, "gdn_decode_fused: one row per sequence");
  const at::cuda::CUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  // RADIANCE_GDN_DECODE_SPLIT=2|4 splits each head's state rows over that many CTAs (more CTAs
  // than Hv at batch 1).  Off by default: on the 27B decode step (48 heads, PDL on) it measured
  // 220.6 tok/s with 4 CTAs per head against 221.8 with one, since the kernel sits on the step's
  // dependency chain and not on bandwidth.  Sizes whose grid is small still exercise it in tests.
  static const int ns_env = [] {
    const char* v = std::getenv("RADIANCE_GDN_DECODE_SPLIT");
    return v ? std::atoi(v) : -1;
  }();
  // split: 1 | 2 | 4 CTAs per head, 0 = RADIANCE_GDN_DECODE_SPLIT (default 1; its value 0 sizes
  // the split to the grid)
  const bool fused_q = q.defined() && q.numel();
  const int req = split == 1 || split == 2 || split == 4 ? (int)split : ns_env;
  const int ns = fused_q ? 1
               : req == 1 || req == 2 || req == 4 ? req
               : req == -1 ? 1 : (B * Hv >= 148 ? 1 : B * Hv * 2 >= 148 ? 2 : 4);
  gdn::GdnQuantArgs fq{};
  if (fused_q) {
    TORCH_CHECK(q.scalar_type() == at::kFloat8_e4m3fn && q.size(0) >= B && q.size(1) >= Hv * 128 &&
                    q.stride(1) == 1 && q.stride(0) % 8 == 0, "gdn_decode_fused: q");
    TORCH_CHECK(nout.scalar_type() == at::kBFloat16 && nout.is_contiguous() &&
                    nout.numel() >= (int64_t)B * Hv * 128, "gdn_decode_fused: nout");
    // fixed layout whatever B is: counters [0, 4096) (must stay zero between calls), then the
    // head amax slots (written each call)
    TORCH_CHECK(B <= 4096 && ws.scalar_type() == at::kInt && ws.numel() >= 4096 + (int64_t)B * Hv,
                "gdn ws");
    TORCH_CHECK(norm_w.scalar_type() == at::kBFloat16 && norm_w.numel() >= 128, "norm weight");
    TORCH_CHECK(q_scale.scalar_type() == at::kFloat && q_scale.numel() >= B, "q_scale");
    fq.z_off = (int)z_off;
    fq.norm_w = (const __nv_bfloat16*)norm_w.data_ptr();
    fq.norm_eps = (float)norm_eps;
    fq.nout = (__nv_bfloat16*)nout.data_ptr();
    fq.row_cnt = reinterpret_cast<unsigned*>(ws.data_ptr<int>());
    fq.head_amax = reinterpret_cast<float*>(ws.data_ptr<int>() + 4096);
    fq.q = (uint8_t*)q.data_ptr();
    fq.ldq = (int)q.stride(0);
    fq.q_scale = q_scale.data_ptr<float>();
  }
  auto run = [&](auto stag) {
    using ST = typename decltype(stag)::type;
    auto kern = fused_q ? gdn::decode_fused_kernel<128, ST, 1, true>
              : ns == 4 ? gdn::decode_fused_kernel<128, ST, 4>
              : ns == 2 ? gdn::decode_fused_kernel<128, ST, 2> : gdn::decode_fused_kernel<128, ST, 1>;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(B, Hv, ns);
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeClusterDimension;
    attrs[0].val.clusterDim.x = 1;
    attrs[0].val.clusterDim.y = Hv / Hk;
    attrs[0].val.clusterDim.z = 1;
    attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, (const __nv_bfloat16*)x.data_ptr(),
        (int)x.stride(0), (const __nv_bfloat16*)conv_w.data_ptr(),
        (__nv_bfloat16*)conv_state.data_ptr(), (int)ba_off, A_log.data_ptr<float>(),
        dt_bias.data_ptr<float>(), (ST*)state.data_ptr(), slots.data_ptr<int>(),
        has_init.data_ptr<int>(), (int)Hk, Hv, C, (float)scale, (float)eps,
        fused_q ? nullptr : (__nv_bfloat16*)out.data_ptr(), fused_q ? 0 : (int)out.stride(0), fq));
  };
  struct F32 { using type = float; };
  struct BF16 { using type = __nv_bfloat16; };
  if (state.scalar_type() == at::kFloat) run(F32{});
  else run(BF16{});
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace rad
