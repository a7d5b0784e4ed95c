// Chunked gated-delta-rule prefill (the one-round chunk scan of the GDN layers).
//
// Reference behaviour: libr4d gdn_kkt_solve + gdn_chunk_scan_k128_v128_c64 (radiance_gdn.py:
// 510-560, sly/r4d/r4d_gdn_scan_variants.patch, exact-decay form sly/r4d/r4d_gdn_exact_decay.patch)
// with the oracle sly/gdn/chunk_scan_ref.py:71-110.  Same math as the token-serial recurrence
//   S_t = e^{g_t} S_{t-1} + beta_t (v_t - e^{g_t} S_{t-1} k_t) k_t^T,   o_t = scale * S_t q_t
// evaluated 64 tokens at a time.  Per chunk, with G = in-chunk cumulative sum of g:
//   A   = strict_lower(beta_i (k_i . k_j) e^{G_i - G_j})                 [64 x 64]
//   P   = lower(q_i . k_j e^{G_i - G_j})   (diagonal included)           [64 x 64]
//   RHS = beta (V - e^{G} K S^T)                                          [64 x dv]
//   (I + A) U = RHS                        (blocked forward substitution, 16-row blocks)
//   O   = scale (e^{G} Q S^T + P U)
//   S  <- e^{G_last} S + (e^{G_last - G} U)^T K
//
// B200 design: one CTA of 8 warps per (sequence, value head) walks the sequence chunk by chunk.
// All matrix products run on the tensor cores as bf16 mma.sync with fp32 accumulation; operand
// tiles live in shared memory (XOR-swizzled 16-byte chunks, ldmatrix).  The fp32 state stays in
// registers for the whole sequence (warp w owns rows [16w, 16w + 16) of S), and a bf16 copy in
// shared memory feeds the K S^T / Q S^T products.  The triangular solve is organised so that
// every warp owns 16 value columns end to end: no CTA barrier inside it.
//
// Head dims dk = dv = 128 (the production geometry); other sizes use the token-serial kernel.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace rad {
namespace gdnc {

constexpr int D = 128;          // dk = dv
constexpr int C = 64;           // chunk length
constexpr int CHD = D / 8;      // 16-byte chunks per D-wide bf16 row
constexpr int CHC = C / 8;      // 16-byte chunks per C-wide bf16 row
constexpr int kThreads = 256;

// shared-memory map (bytes)
constexpr int OFF_K = 0;                          // [C][D] bf16
constexpr int OFF_Q = OFF_K + C * D * 2;          // [C][D] bf16
constexpr int OFF_V = OFF_Q + C * D * 2;          // [C][D] bf16
constexpr int OFF_S = OFF_V + C * D * 2;          // [D][D] bf16 (state copy, [dv][dk])
constexpr int OFF_R = OFF_S + D * D * 2;          // [C][D] bf16 RHS
constexpr int OFF_U = OFF_R + C * D * 2;          // [C][D] bf16 U
constexpr int OFF_US = OFF_U + C * D * 2;         // [C][D] bf16 e^{G_last - G} U
constexpr int OFF_A = OFF_US + C * D * 2;         // [C][C] fp32 A
constexpr int OFF_AB = OFF_A + C * C * 4;         // [C][C] bf16 A
constexpr int OFF_P = OFF_AB + C * C * 2;         // [C][C] bf16 P
constexpr int OFF_T = OFF_P + C * C * 2;          // [4][16][16] bf16 diagonal-block inverses
constexpr int OFF_X = OFF_T + 4 * 16 * 16 * 2;    // [16][D] bf16 solve scratch
constexpr int OFF_G = OFF_X + 16 * D * 2;         // [C] fp32 cumulative log decay
constexpr int OFF_B = OFF_G + C * 4;              // [C] fp32 beta
constexpr int SMEM = OFF_B + C * 4;

DEVI uint32_t swz(int row, int chunk, int ch) {
  return (uint32_t)(row * ch + (chunk ^ (row & 7))) * 16u;
}
DEVI void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
DEVI void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
DEVI void mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// A fragment (16 x 16) from a row-major [rows][k] tile; kc = first k chunk (k0 / 8)
DEVI void ldA(uint32_t base, int row0, int kc, int ch, int lane, uint32_t (&a)[4]) {
  ldsm_x4(base + swz(row0 + (lane & 15), kc + (lane >> 4), ch), a);
}
// A fragment of X^T from a row-major [k][m] tile; mc = first m chunk (m0 / 8)
DEVI void ldAt(uint32_t base, int k0, int mc, int ch, int lane, uint32_t (&a)[4]) {
  ldsm_x4_t(base + swz(k0 + (lane & 7) + (lane >> 4) * 8, mc + ((lane >> 3) & 1), ch), a);
}
// B fragments of n-tiles (n0, n0 + 8) from a row-major [n][k] tile
DEVI void ldB(uint32_t base, int n0, int kc, int ch, int lane, uint32_t (&b)[4]) {
  ldsm_x4(base + swz(n0 + (lane & 7) + (lane >> 4) * 8, kc + ((lane >> 3) & 1), ch), b);
}
// B fragments of n-tiles (n0, n0 + 8) from a row-major [k][n] tile; nc = n0 / 8
DEVI void ldBt(uint32_t base, int k0, int nc, int ch, int lane, uint32_t (&b)[4]) {
  ldsm_x4_t(base + swz(k0 + (lane & 7) + ((lane >> 3) & 1) * 8, nc + (lane >> 4), ch), b);
}
DEVI void st_bf16x2(uint8_t* base, int row, int col, int ch, float x, float y) {
  __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
  *reinterpret_cast<__nv_bfloat162*>(base + swz(row, col >> 3, ch) + (col & 7) * 2) = h;
}
DEVI float2 ld_bf16x2(const uint8_t* base, int row, int col, int ch) {
  return __bfloat1622float2(
      *reinterpret_cast<const __nv_bfloat162*>(base + swz(row, col >> 3, ch) + (col & 7) * 2));
}

// NS CTAs share one (sequence, head): CTA z owns value columns [z * 128 / NS, (z + 1) * 128 / NS)
// of V, RHS, U, O and the matching rows of S; the intra-chunk K K^T / Q K^T terms are computed
// by each of them (small next to the per-column work), so no data crosses CTAs.
template <typename ST, int NS>
__global__ void __launch_bounds__(kThreads, 1) chunk_kernel(
    const __nv_bfloat16* __restrict__ y, int ldy,        // conv output [T, *]: q | k | v
    const __nv_bfloat16* __restrict__ ba, int ldba,      // [T, *]: b at col 0.., a at col Hv..
    const float* __restrict__ A_log, const float* __restrict__ dt_bias,
    ST* __restrict__ state,                              // [S, Hv, D, D]
    const int* __restrict__ qsl, const int* __restrict__ slots, const int* __restrict__ has_init,
    int Hk, int Hv, float scale, __nv_bfloat16* __restrict__ out, int ldo) {
  pdl_wait();     // inputs come from the preceding kernel
  pdl_trigger();
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sK = smem + OFF_K;
  uint8_t* sQ = smem + OFF_Q;
  uint8_t* sV = smem + OFF_V;
  uint8_t* sS = smem + OFF_S;
  uint8_t* sR = smem + OFF_R;
  uint8_t* sU = smem + OFF_U;
  uint8_t* sUs = smem + OFF_US;
  float* sA = reinterpret_cast<float*>(smem + OFF_A);
  uint8_t* sAb = smem + OFF_AB;
  uint8_t* sP = smem + OFF_P;
  uint8_t* sT = smem + OFF_T;
  uint8_t* sX = smem + OFF_X;
  float* sG = reinterpret_cast<float*>(smem + OFF_G);
  float* sBeta = reinterpret_cast<float*>(smem + OFF_B);
  const uint32_t aK = smem_u32(sK), aQ = smem_u32(sQ), aS = smem_u32(sS), aR = smem_u32(sR);
  const uint32_t aU = smem_u32(sU), aUs = smem_u32(sUs), aAb = smem_u32(sAb), aP = smem_u32(sP);
  const uint32_t aT = smem_u32(sT), aX = smem_u32(sX);

  constexpr int DVS = D / NS;                       // value columns of this CTA
  const int b = blockIdx.x, h = blockIdx.y;
  const int voff = blockIdx.z * DVS;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g_ = lane >> 2, t4 = lane & 3;
  const int s0 = qsl[b];
  const int L = qsl[b + 1] - s0;
  if (L <= 0) return;
  const int slot = slots[b];
  const int hk = h / (Hv / Hk);
  const int key_dim = Hk * D;
  const float negA = -__expf(A_log[h]);
  const float dtb = dt_bias[h];

  // ---- state: fp32 in registers.  Rows [voff, voff + DVS) of S [dv][dk] belong to this CTA:
  //      warp w owns the 16-row block w / NS and dk columns [(w % NS) * 128 / NS, ...) ----
  constexpr int SNT = 16 / NS;                       // 8-wide dk tiles per warp
  const int srow = voff + 16 * (warp / NS);
  const int scol = (warp % NS) * (D / NS);
  float Sr[SNT][4];
  ST* gS = state + ((size_t)slot * Hv + h) * D * D;
  const bool init = has_init[b] != 0;
#pragma unroll
  for (int n = 0; n < SNT; ++n) {
    const int r0 = srow + g_, c = scol + n * 8 + 2 * t4;
    Sr[n][0] = init ? to_f(gS[(size_t)r0 * D + c]) : 0.f;
    Sr[n][1] = init ? to_f(gS[(size_t)r0 * D + c + 1]) : 0.f;
    Sr[n][2] = init ? to_f(gS[(size_t)(r0 + 8) * D + c]) : 0.f;
    Sr[n][3] = init ? to_f(gS[(size_t)(r0 + 8) * D + c + 1]) : 0.f;
    st_bf16x2(sS, r0, c, CHD, Sr[n][0], Sr[n][1]);
    st_bf16x2(sS, r0 + 8, c, CHD, Sr[n][2], Sr[n][3]);
  }

  for (int c0 = 0; c0 < L; c0 += C) {
    const int m = min(C, L - c0);
    __syncthreads();            // previous chunk is done with every tile
    // ---- load K, Q, V rows of the chunk (zero past the end) ----
    for (int idx = threadIdx.x; idx < 3 * C * CHD; idx += kThreads) {
      const int which = idx / (C * CHD), rem = idx % (C * CHD);
      const int r = rem / CHD, ch = rem % CHD;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (r < m) {
        const __nv_bfloat16* row = y + (size_t)(s0 + c0 + r) * ldy;
        const int col = which == 0 ? key_dim + hk * D : which == 1 ? hk * D : 2 * key_dim + h * D;
        v = *reinterpret_cast<const uint4*>(row + col + ch * 8);
      }
      uint8_t* dst = which == 0 ? sK : which == 1 ? sQ : sV;
      *reinterpret_cast<uint4*>(dst + swz(r, ch, CHD)) = v;
    }
    // ---- gates + in-chunk cumulative log decay (warp 0: two tokens per lane) ----
    if (warp == 0) {
      float gl[2], bl[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int r = lane * 2 + e;
        gl[e] = 0.f;
        bl[e] = 0.f;
        if (r < m) {
          const size_t t = s0 + c0 + r;
          const float bb = __bfloat162float(ba[t * ldba + h]);
          const float aa = __bfloat162float(ba[t * ldba + Hv + h]);
          const float xs = aa + dtb;
          const float sp = xs > 20.f ? xs : log1pf(__expf(xs));
          gl[e] = negA * sp;
          bl[e] = 1.f / (1.f + __expf(-bb));
        }
      }
      float pair = gl[0] + gl[1];
      float incl = pair;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      const float excl = incl - pair;
      sG[lane * 2] = excl + gl[0];
      sG[lane * 2 + 1] = incl;
      sBeta[lane * 2] = bl[0];
      sBeta[lane * 2 + 1] = bl[1];
    }
    __syncthreads();
    const float Glast = sG[C - 1];

    // ---- A = strict_lower(beta K K^T e^{dG}),  P = lower(Q K^T e^{dG}) ----
    {
      const int mt = warp >> 1;               // 16-row block of the chunk
      const int nb = (warp & 1) * 32;         // 32 key columns
      float ak[4][4], ap[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) ak[j][e] = ap[j][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        uint32_t fk[4], fq[4];
        ldA(aK, 16 * mt, 2 * kk, CHD, lane, fk);
        ldA(aQ, 16 * mt, 2 * kk, CHD, lane, fq);
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          uint32_t bk[4];
          ldB(aK, nb + 16 * np, 2 * kk, CHD, lane, bk);
          mma(ak[2 * np], fk, bk[0], bk[1]);
          mma(ak[2 * np + 1], fk, bk[2], bk[3]);
          mma(ap[2 * np], fq, bk[0], bk[1]);
          mma(ap[2 * np + 1], fq, bk[2], bk[3]);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int i = 16 * mt + g_ + 8 * hh;
          const int c = nb + 8 * j + 2 * t4;
          const float Gi = sG[i], bi = sBeta[i];
          float av[2], pv[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int jj = c + e;
            const float d = __expf(fminf(Gi - sG[jj], 0.f));
            av[e] = jj < i ? bi * ak[j][2 * hh + e] * d : 0.f;
            pv[e] = jj <= i ? ap[j][2 * hh + e] * d : 0.f;
          }
          sA[i * C + c] = av[0];
          sA[i * C + c + 1] = av[1];
          st_bf16x2(sAb, i, c, CHC, av[0], av[1]);
          st_bf16x2(sP, i, c, CHC, pv[0], pv[1]);
        }
      }
    }

    // ---- K S^T and Q S^T: RHS = beta (V - e^G K S^T); O = e^G Q S^T (kept in registers) ----
    constexpr int ONT = DVS / 16;            // 8-wide value tiles per warp in the [64 x DVS] stages
    float o[ONT][4];
    {
      const int mt = warp >> 1;
      const int nb = voff + (warp & 1) * (DVS / 2);
      float ks[ONT][4];
#pragma unroll
      for (int j = 0; j < ONT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) ks[j][e] = o[j][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        uint32_t fk[4], fq[4];
        ldA(aK, 16 * mt, 2 * kk, CHD, lane, fk);
        ldA(aQ, 16 * mt, 2 * kk, CHD, lane, fq);
#pragma unroll
        for (int np = 0; np < ONT / 2; ++np) {
          uint32_t bs[4];
          ldB(aS, nb + 16 * np, 2 * kk, CHD, lane, bs);
          mma(ks[2 * np], fk, bs[0], bs[1]);
          mma(ks[2 * np + 1], fk, bs[2], bs[3]);
          mma(o[2 * np], fq, bs[0], bs[1]);
          mma(o[2 * np + 1], fq, bs[2], bs[3]);
        }
      }
#pragma unroll
      for (int j = 0; j < ONT; ++j) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int i = 16 * mt + g_ + 8 * hh;
          const int c = nb + 8 * j + 2 * t4;
          const float eg = __expf(sG[i]), bi = sBeta[i];
          const float2 v = ld_bf16x2(sV, i, c, CHD);
          st_bf16x2(sR, i, c, CHD, bi * (v.x - eg * ks[j][2 * hh]), bi * (v.y - eg * ks[j][2 * hh + 1]));
          o[j][2 * hh] *= eg;
          o[j][2 * hh + 1] *= eg;
        }
      }
    }
    __syncthreads();

    // ---- inverses of the four unit-lower diagonal blocks of (I + A): warps 0-3, lane = column ----
    if (warp < 4 && lane < 16) {
      const int bo = 16 * warp;
      float t[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float acc = (i == lane) ? 1.f : 0.f;
#pragma unroll
        for (int j = 0; j < i; ++j) acc -= sA[(bo + i) * C + bo + j] * t[j];
        t[i] = acc;
      }
      __nv_bfloat16* T = reinterpret_cast<__nv_bfloat16*>(sT) + warp * 256;
#pragma unroll
      for (int i = 0; i < 16; ++i) T[i * 16 + lane] = __float2bfloat16_rn(t[i]);
    }
    __syncthreads();

    // ---- (I + A) U = RHS, blocked: warp w owns value columns voff + [16w, 16w + 16) ----
    if (warp < DVS / 16) {
      const int nc = (voff >> 3) + 2 * warp;  // first 8-column chunk of this warp
#pragma unroll
      for (int bi = 0; bi < 4; ++bi) {
        float x[2][4];
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) x[j][e] = 0.f;
        for (int kk = 0; kk < bi; ++kk) {     // sum_{k < bi} A_{bi,k} U_k
          uint32_t fa[4], bu[4];
          ldA(aAb, 16 * bi, 2 * kk, CHC, lane, fa);
          ldBt(aU, 16 * kk, nc, CHD, lane, bu);
          mma(x[0], fa, bu[0], bu[1]);
          mma(x[1], fa, bu[2], bu[3]);
        }
        // X = RHS_bi - sum  -> scratch (this warp's columns only)
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int c = 8 * (nc + j) + 2 * t4;
            const float2 r = ld_bf16x2(sR, 16 * bi + g_ + 8 * hh, c, CHD);
            st_bf16x2(sX, g_ + 8 * hh, c, CHD, r.x - x[j][2 * hh], r.y - x[j][2 * hh + 1]);
          }
        __syncwarp();
        // U_bi = T_bi X
        uint32_t ft[4], bx[4];
        ldsm_x4(aT + bi * 512 + ((lane & 15) * 2 + (lane >> 4)) * 16, ft);
        ldBt(aX, 0, nc, CHD, lane, bx);
        float u[2][4];
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) u[j][e] = 0.f;
        mma(u[0], ft, bx[0], bx[1]);
        mma(u[1], ft, bx[2], bx[3]);
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int i = 16 * bi + g_ + 8 * hh;
            const int c = 8 * (nc + j) + 2 * t4;
            const float ds = __expf(Glast - sG[i]);
            st_bf16x2(sU, i, c, CHD, u[j][2 * hh], u[j][2 * hh + 1]);
            st_bf16x2(sUs, i, c, CHD, u[j][2 * hh] * ds, u[j][2 * hh + 1] * ds);
          }
        __syncwarp();
      }
    }
    __syncthreads();

    // ---- O += P U; write the chunk's outputs ----
    {
      const int mt = warp >> 1;
      const int nb = voff + (warp & 1) * (DVS / 2);
#pragma unroll
      for (int kk = 0; kk < C / 16; ++kk) {
        uint32_t fp[4];
        ldA(aP, 16 * mt, 2 * kk, CHC, lane, fp);
#pragma unroll
        for (int np = 0; np < ONT / 2; ++np) {
          uint32_t bu[4];
          ldBt(aU, 16 * kk, (nb >> 3) + 2 * np, CHD, lane, bu);
          mma(o[2 * np], fp, bu[0], bu[1]);
          mma(o[2 * np + 1], fp, bu[2], bu[3]);
        }
      }
#pragma unroll
      for (int j = 0; j < ONT; ++j)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int i = 16 * mt + g_ + 8 * hh;
          if (i < m) {
            const int c = nb + 8 * j + 2 * t4;
            *reinterpret_cast<__nv_bfloat162*>(out + (size_t)(s0 + c0 + i) * ldo + h * D + c) =
                __floats2bfloat162_rn(scale * o[j][2 * hh], scale * o[j][2 * hh + 1]);
          }
        }
    }

    // ---- S <- e^{G_last} S + (e^{G_last - G} U)^T K;  refresh the bf16 copy ----
    {
      float acc[SNT][4];
#pragma unroll
      for (int n = 0; n < SNT; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < C / 16; ++kk) {
        uint32_t fu[4];
        ldAt(aUs, 16 * kk, srow >> 3, CHD, lane, fu);
#pragma unroll
        for (int np = 0; np < SNT / 2; ++np) {
          uint32_t bk[4];
          ldBt(aK, 16 * kk, (scol >> 3) + 2 * np, CHD, lane, bk);
          mma(acc[2 * np], fu, bk[0], bk[1]);
          mma(acc[2 * np + 1], fu, bk[2], bk[3]);
        }
      }
      const float dl = __expf(Glast);
      __syncthreads();          // every warp has finished reading the previous bf16 state
#pragma unroll
      for (int n = 0; n < SNT; ++n) {
        const int r0 = srow + g_, c = scol + n * 8 + 2 * t4;
#pragma unroll
        for (int e = 0; e < 4; ++e) Sr[n][e] = dl * Sr[n][e] + acc[n][e];
        st_bf16x2(sS, r0, c, CHD, Sr[n][0], Sr[n][1]);
        st_bf16x2(sS, r0 + 8, c, CHD, Sr[n][2], Sr[n][3]);
      }
    }
  }

  // ---- final state ----
#pragma unroll
  for (int n = 0; n < SNT; ++n) {
    const int r0 = srow + g_, c = scol + n * 8 + 2 * t4;
    gS[(size_t)r0 * D + c] = from_f<ST>(Sr[n][0]);
    gS[(size_t)r0 * D + c + 1] = from_f<ST>(Sr[n][1]);
    gS[(size_t)(r0 + 8) * D + c] = from_f<ST>(Sr[n][2]);
    gS[(size_t)(r0 + 8) * D + c + 1] = from_f<ST>(Sr[n][3]);
  }
}


// =============================================================================================
// Two-phase form.  The state-dependent part of a chunk only needs terms that do not depend on S:
//   W  = (I + A)^{-1} diag(beta e^G) K        [64 x dk]
//   U0 = (I + A)^{-1} diag(beta) V            [64 x dv]
// because U = (I + A)^{-1} beta (V - e^G K S^T) = U0 - W S^T.  Phase 1 (prep_kernel) solves W,
// U0 and forms P and G for every (chunk, value head) at once -- all chunks in parallel.  Phase 2
// (scan_kernel) walks the chunks of one (sequence, head, value slice) with three small products
// per chunk and no triangular solve, so the value dimension splits 2, 4 or 8 ways without
// repeating the solve (the one-kernel form above repeats K K^T and the solve in every slice).
// =============================================================================================
constexpr int WS_W = 0;                        // [C][D] bf16   W
constexpr int WS_U = WS_W + C * D * 2;         // [C][D] bf16   U0
constexpr int WS_P = WS_U + C * D * 2;         // [C][C] bf16   P
constexpr int WS_G = WS_P + C * C * 2;         // [C]    fp32   G
constexpr int WS_CHUNK = WS_G + C * 4;         // bytes per (chunk, value head)

constexpr int CH2 = 2 * D / 8;                 // 16-byte chunks of a [.][2D] bf16 row
// phase-1 shared memory (two CTAs per SM)
constexpr int Q1_K = 0;                        // [C][D] bf16
constexpr int Q1_Q = Q1_K + C * D * 2;         // [C][D] bf16
constexpr int Q1_R = Q1_Q + C * D * 2;         // [C][2D] bf16 right-hand sides, solved in place
constexpr int Q1_AD = Q1_R + C * 2 * D * 2;    // [4][16][16] fp32 diagonal blocks of A
constexpr int Q1_AB = Q1_AD + 4 * 256 * 4;     // [C][C] bf16 A
constexpr int Q1_T = Q1_AB + C * C * 2;        // [4][16][16] bf16 diagonal-block inverses
constexpr int Q1_X = Q1_T + 4 * 256 * 2;       // [16][2D] bf16 solve scratch
constexpr int Q1_G = Q1_X + 16 * 2 * D * 2;    // [C] fp32
constexpr int Q1_B = Q1_G + C * 4;             // [C] fp32
constexpr int SMEM1 = Q1_B + C * 4;

// chunk x of the flattened batch -> (sequence, first token of the chunk); false past the end
DEVI bool chunk_of(const int* __restrict__ qsl, int B, int x, int& b, int& c0) {
  int acc = 0;
  for (int i = 0; i < B; ++i) {
    const int n = (qsl[i + 1] - qsl[i] + C - 1) / C;
    if (x < acc + n) {
      b = i;
      c0 = (x - acc) * C;
      return true;
    }
    acc += n;
  }
  return false;
}

// gates of the 64 tokens [c0, c0 + m) of a sequence starting at s0: in-chunk cumulative log
// decay G and beta (warp 0; two tokens per lane; zero past m)
DEVI void chunk_gates(const __nv_bfloat16* __restrict__ ba, int ldba, int Hv, int h, float negA,
                      float dtb, int s0, int c0, int m, int lane, float* sG, float* sBeta) {
  float gl[2], bl[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int r = lane * 2 + e;
    gl[e] = 0.f;
    bl[e] = 0.f;
    if (r < m) {
      const size_t t = s0 + c0 + r;
      const float bb = __bfloat162float(ba[t * ldba + h]);
      const float aa = __bfloat162float(ba[t * ldba + Hv + h]);
      const float xs = aa + dtb;
      const float sp = xs > 20.f ? xs : log1pf(__expf(xs));
      gl[e] = negA * sp;
      bl[e] = 1.f / (1.f + __expf(-bb));
    }
  }
  const float pair = gl[0] + gl[1];
  float incl = pair;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  const float excl = incl - pair;
  sG[lane * 2] = excl + gl[0];
  sG[lane * 2 + 1] = incl;
  sBeta[lane * 2] = bl[0];
  sBeta[lane * 2 + 1] = bl[1];
}

// Phase 1: one CTA per (chunk of the flattened batch, value head).
__global__ void __launch_bounds__(kThreads, 2) prep_kernel(
    const __nv_bfloat16* __restrict__ y, int ldy, const __nv_bfloat16* __restrict__ ba, int ldba,
    const float* __restrict__ A_log, const float* __restrict__ dt_bias,
    const int* __restrict__ qsl, int B, int Hk, int Hv, uint8_t* __restrict__ ws) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sK = smem + Q1_K;
  uint8_t* sQ = smem + Q1_Q;
  uint8_t* sR = smem + Q1_R;
  float* sAD = reinterpret_cast<float*>(smem + Q1_AD);
  uint8_t* sAb = smem + Q1_AB;
  uint8_t* sT = smem + Q1_T;
  uint8_t* sX = smem + Q1_X;
  float* sG = reinterpret_cast<float*>(smem + Q1_G);
  float* sBeta = reinterpret_cast<float*>(smem + Q1_B);
  const uint32_t aK = smem_u32(sK), aQ = smem_u32(sQ), aR = smem_u32(sR), aAb = smem_u32(sAb);
  const uint32_t aT = smem_u32(sT), aX = smem_u32(sX);
  const int h = blockIdx.y;
  int b, c0;
  if (!chunk_of(qsl, B, blockIdx.x, b, c0)) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g_ = lane >> 2, t4 = lane & 3;
  const int s0 = qsl[b];
  const int m = min(C, qsl[b + 1] - s0 - c0);
  const int hk = h / (Hv / Hk);
  const int key_dim = Hk * D;
  uint8_t* wsc = ws + ((size_t)blockIdx.x * Hv + h) * WS_CHUNK;

  // ---- K, Q and (into the right half of R) V rows of the chunk, zero past m ----
  for (int idx = threadIdx.x; idx < 3 * C * CHD; idx += kThreads) {
    const int which = idx / (C * CHD), rem = idx % (C * CHD);
    const int r = rem / CHD, ch = rem % CHD;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < m) {
      const __nv_bfloat16* row = y + (size_t)(s0 + c0 + r) * ldy;
      const int col = which == 0 ? key_dim + hk * D : which == 1 ? hk * D : 2 * key_dim + h * D;
      v = *reinterpret_cast<const uint4*>(row + col + ch * 8);
    }
    uint8_t* dst = which == 0 ? sK + swz(r, ch, CHD) : which == 1 ? sQ + swz(r, ch, CHD)
                                                                  : sR + swz(r, CHD + ch, CH2);
    *reinterpret_cast<uint4*>(dst) = v;
  }
  if (warp == 0)
    chunk_gates(ba, ldba, Hv, h, -__expf(A_log[h]), dt_bias[h], s0, c0, m, lane, sG, sBeta);
  __syncthreads();
  if (threadIdx.x < C) reinterpret_cast<float*>(wsc + WS_G)[threadIdx.x] = sG[threadIdx.x];

  // ---- right-hand sides: R = [beta e^G K | beta V] ----
  for (int idx = threadIdx.x; idx < C * CH2; idx += kThreads) {
    const int r = idx / CH2, ch = idx % CH2;
    const float f = ch < CHD ? sBeta[r] * __expf(sG[r]) : sBeta[r];
    const uint4 u = *reinterpret_cast<const uint4*>(ch < CHD ? sK + swz(r, ch, CHD)
                                                             : sR + swz(r, ch, CH2));
    uint4 o;
    const __nv_bfloat162* hi = reinterpret_cast<const __nv_bfloat162*>(&u);
    __nv_bfloat162* ho = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 t = __bfloat1622float2(hi[k]);
      ho[k] = __floats2bfloat162_rn(t.x * f, t.y * f);
    }
    *reinterpret_cast<uint4*>(sR + swz(r, ch, CH2)) = o;
  }

  // ---- A = strict_lower(beta K K^T e^{dG}) (bf16, diagonal blocks also fp32);
  //      P = lower(Q K^T e^{dG}) straight to the workspace ----
  {
    const int mt = warp >> 1;               // 16-row block of the chunk
    const int nb = (warp & 1) * 32;         // 32 key columns
    float ak[4][4], ap[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) ak[j][e] = ap[j][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t fk[4], fq[4];
      ldA(aK, 16 * mt, 2 * kk, CHD, lane, fk);
      ldA(aQ, 16 * mt, 2 * kk, CHD, lane, fq);
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        uint32_t bk[4];
        ldB(aK, nb + 16 * np, 2 * kk, CHD, lane, bk);
        mma(ak[2 * np], fk, bk[0], bk[1]);
        mma(ak[2 * np + 1], fk, bk[2], bk[3]);
        mma(ap[2 * np], fq, bk[0], bk[1]);
        mma(ap[2 * np + 1], fq, bk[2], bk[3]);
      }
    }
    __nv_bfloat16* gP = reinterpret_cast<__nv_bfloat16*>(wsc + WS_P);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int i = 16 * mt + g_ + 8 * hh;
        const int c = nb + 8 * j + 2 * t4;
        const float Gi = sG[i], bi = sBeta[i];
        float av[2], pv[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int jj = c + e;
          const float d = __expf(fminf(Gi - sG[jj], 0.f));
          av[e] = jj < i ? bi * ak[j][2 * hh + e] * d : 0.f;
          pv[e] = jj <= i ? ap[j][2 * hh + e] * d : 0.f;
          if ((jj >> 4) == (i >> 4)) sAD[(i >> 4) * 256 + (i & 15) * 16 + (jj & 15)] = av[e];
        }
        st_bf16x2(sAb, i, c, CHC, av[0], av[1]);
        *reinterpret_cast<__nv_bfloat162*>(gP + i * C + c) = __floats2bfloat162_rn(pv[0], pv[1]);
      }
    }
  }
  __syncthreads();

  // ---- inverses of the four unit-lower diagonal blocks of (I + A): warps 0-3, lane = column ----
  if (warp < 4 && lane < 16) {
    const float* Ad = sAD + warp * 256;
    float t[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float acc = (i == lane) ? 1.f : 0.f;
#pragma unroll
      for (int j = 0; j < i; ++j) acc -= Ad[i * 16 + j] * t[j];
      t[i] = acc;
    }
    __nv_bfloat16* T = reinterpret_cast<__nv_bfloat16*>(sT) + warp * 256;
#pragma unroll
    for (int i = 0; i < 16; ++i) T[i * 16 + lane] = __float2bfloat16_rn(t[i]);
  }
  __syncthreads();

  // ---- (I + A) [W | U0] = R in place, blocked: warp w owns columns [32w, 32w + 32) ----
  {
    const int nc0 = 4 * warp;               // first 8-column chunk of this warp
#pragma unroll
    for (int bi = 0; bi < 4; ++bi) {
      float x[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) x[j][e] = 0.f;
      for (int kk = 0; kk < bi; ++kk) {     // sum_{k < bi} A_{bi,k} Y_k (rows kk already solved)
        uint32_t fa[4];
        ldA(aAb, 16 * bi, 2 * kk, CHC, lane, fa);
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          uint32_t bu[4];
          ldBt(aR, 16 * kk, nc0 + 2 * np, CH2, lane, bu);
          mma(x[2 * np], fa, bu[0], bu[1]);
          mma(x[2 * np + 1], fa, bu[2], bu[3]);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int c = 8 * (nc0 + j) + 2 * t4;
          const float2 r = ld_bf16x2(sR, 16 * bi + g_ + 8 * hh, c, CH2);
          st_bf16x2(sX, g_ + 8 * hh, c, CH2, r.x - x[j][2 * hh], r.y - x[j][2 * hh + 1]);
        }
      __syncwarp();
      uint32_t ft[4];
      ldsm_x4(aT + bi * 512 + ((lane & 15) * 2 + (lane >> 4)) * 16, ft);
      float u[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) u[j][e] = 0.f;
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        uint32_t bx[4];
        ldBt(aX, 0, nc0 + 2 * np, CH2, lane, bx);
        mma(u[2 * np], ft, bx[0], bx[1]);
        mma(u[2 * np + 1], ft, bx[2], bx[3]);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int c = 8 * (nc0 + j) + 2 * t4;
          st_bf16x2(sR, 16 * bi + g_ + 8 * hh, c, CH2, u[j][2 * hh], u[j][2 * hh + 1]);
        }
      __syncwarp();
    }
  }
  __syncthreads();

  // ---- W | U0 to the workspace (row-major [C][D] each) ----
  for (int idx = threadIdx.x; idx < C * CH2; idx += kThreads) {
    const int r = idx / CH2, ch = idx % CH2;
    const uint4 v = *reinterpret_cast<const uint4*>(sR + swz(r, ch, CH2));
    uint8_t* dst = wsc + (ch < CHD ? WS_W + (r * D + ch * 8) * 2 : WS_U + (r * D + (ch - CHD) * 8) * 2);
    *reinterpret_cast<uint4*>(dst) = v;
  }
}

DEVI void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(valid ? 16 : 0) : "memory");
}
DEVI void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
DEVI void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// phase-2 stage: the chunk's W, Q, K (bf16 [C][D]), U0 columns of the slice ([C][64] bf16, first
// DVS used), P ([C][C] bf16) and G
constexpr int Q2_W = 0;
constexpr int Q2_Q = Q2_W + C * D * 2;
constexpr int Q2_K = Q2_Q + C * D * 2;
constexpr int Q2_U0 = Q2_K + C * D * 2;
constexpr int Q2_P = Q2_U0 + C * 64 * 2;
constexpr int Q2_G = Q2_P + C * C * 2;
constexpr int Q2_STAGE = Q2_G + C * 4;
constexpr int CH64 = 8;                        // 16-byte chunks of a [.][64] bf16 row
// after the two stages: bf16 state slice [64][D] (first DVS rows used), U and e^{G_last - G} U
constexpr int Q2_S = 2 * Q2_STAGE;
constexpr int Q2_U = Q2_S + 64 * D * 2;
constexpr int Q2_US = Q2_U + C * 64 * 2;
constexpr int SMEM2 = Q2_US + C * 64 * 2;

// Phase 2: one CTA of 8 warps per (sequence, value head, value slice of DVS = 128 / NS columns).
// Per chunk: warps 0-3 form W S^T and warps 4-7 Q S^T (one 16-row block each); warps 0-3 turn the
// first into U = U0 - W S^T; warps 4-7 add P U and write the outputs while every warp forms its
// part of (e^{G_last - G} U)^T K for the state.  The next chunk's tiles load by cp.async under
// the current chunk's products.
template <typename ST, int NS>
__global__ void __launch_bounds__(kThreads, 1) scan_kernel(
    const __nv_bfloat16* __restrict__ y, int ldy, ST* __restrict__ state,
    const int* __restrict__ qsl, const int* __restrict__ slots, const int* __restrict__ has_init,
    int Hk, int Hv, float scale, const uint8_t* __restrict__ ws, __nv_bfloat16* __restrict__ out,
    int ldo) {
  constexpr int DVS = D / NS;
  static_assert(DVS >= 16 && DVS <= 64, "value slice of 16..64 columns");
  constexpr int ONT = DVS / 8;                 // 8-wide value tiles of a 16-row block
  constexpr int MS = DVS / 16;                 // 16-row blocks of the state slice
  constexpr int SNT = DVS / 8;                 // 8-wide dk tiles per warp in the state update
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(128) uint8_t smem[];
  const int b = blockIdx.x, h = blockIdx.y;
  const int voff = blockIdx.z * DVS;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g_ = lane >> 2, t4 = lane & 3;
  const int s0 = qsl[b];
  const int L = qsl[b + 1] - s0;
  if (L <= 0) return;
  int cbase = 0;
  for (int i = 0; i < b; ++i) cbase += (qsl[i + 1] - qsl[i] + C - 1) / C;
  const int nch = (L + C - 1) / C;
  const int slot = slots[b];
  const int hk = h / (Hv / Hk);
  const int key_dim = Hk * D;
  uint8_t* sS = smem + Q2_S;
  uint8_t* sU = smem + Q2_U;
  uint8_t* sUs = smem + Q2_US;
  const uint32_t aS = smem_u32(sS), aU = smem_u32(sU), aUs = smem_u32(sUs);

  auto load_stage = [&](int j) {
    const int st = j & 1;
    const uint32_t base = smem_u32(smem + st * Q2_STAGE);
    const uint8_t* wsc = ws + ((size_t)(cbase + j) * Hv + h) * WS_CHUNK;
    const int c0 = j * C;
    const int m = min(C, L - c0);
    for (int idx = threadIdx.x; idx < C * CHD; idx += kThreads) {
      const int r = idx / CHD, ch = idx % CHD;
      const uint32_t o = swz(r, ch, CHD);
      cp_async16(base + Q2_W + o, wsc + WS_W + (r * D + ch * 8) * 2, true);
      const __nv_bfloat16* row = y + (size_t)(s0 + c0 + min(r, m - 1)) * ldy;
      cp_async16(base + Q2_Q + o, row + hk * D + ch * 8, r < m);
      cp_async16(base + Q2_K + o, row + key_dim + hk * D + ch * 8, r < m);
    }
    for (int idx = threadIdx.x; idx < C * (DVS / 8); idx += kThreads) {
      const int r = idx / (DVS / 8), ch = idx % (DVS / 8);
      cp_async16(base + Q2_U0 + swz(r, ch, CH64), wsc + WS_U + (r * D + voff + ch * 8) * 2, true);
    }
    for (int idx = threadIdx.x; idx < C * CHC; idx += kThreads) {
      const int r = idx / CHC, ch = idx % CHC;
      cp_async16(base + Q2_P + swz(r, ch, CHC), wsc + WS_P + (r * C + ch * 8) * 2, true);
    }
    if (threadIdx.x < C / 4) cp_async16(base + Q2_G + threadIdx.x * 16, wsc + WS_G + threadIdx.x * 16, true);
    cp_async_commit();
  };

  // ---- state slice: fp32 in registers.  State update tiles: warp w owns the 16-row block
  //      w % MS of the slice and dk columns [(w / MS) * 8 * SNT, ...) ----
  const int srl = 16 * (warp % MS);                 // row of the slice
  const int scol = (warp / MS) * 8 * SNT;
  float Sr[SNT][4];
  ST* gS = state + ((size_t)slot * Hv + h) * D * D;
  const bool init = has_init[b] != 0;
#pragma unroll
  for (int n = 0; n < SNT; ++n) {
    const int r0 = srl + g_, c = scol + n * 8 + 2 * t4;
    const size_t g0 = (size_t)(voff + r0) * D + c, g8 = g0 + 8 * D;
    Sr[n][0] = init ? to_f(gS[g0]) : 0.f;
    Sr[n][1] = init ? to_f(gS[g0 + 1]) : 0.f;
    Sr[n][2] = init ? to_f(gS[g8]) : 0.f;
    Sr[n][3] = init ? to_f(gS[g8 + 1]) : 0.f;
    st_bf16x2(sS, r0, c, CHD, Sr[n][0], Sr[n][1]);
    st_bf16x2(sS, r0 + 8, c, CHD, Sr[n][2], Sr[n][3]);
  }
  load_stage(0);

  const int mt = warp & 3;                          // 16-row block of the chunk (products)
  for (int j = 0; j < nch; ++j) {
    if (j + 1 < nch) {
      load_stage(j + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();                                // stage j landed in every thread's view
    uint8_t* stg = smem + (j & 1) * Q2_STAGE;
    const float* sG = reinterpret_cast<const float*>(stg + Q2_G);
    const uint32_t aW = smem_u32(stg + Q2_W), aQ = smem_u32(stg + Q2_Q), aK = smem_u32(stg + Q2_K);
    const uint32_t aP = smem_u32(stg + Q2_P);
    const int c0 = j * C;
    const int m = min(C, L - c0);
    const float Glast = sG[C - 1];

    // ---- warps 0-3: W S^T, warps 4-7: Q S^T (16 rows x DVS each) ----
    float acc[ONT][4];
#pragma unroll
    for (int n = 0; n < ONT; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
    {
      const uint32_t aA = warp < 4 ? aW : aQ;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        uint32_t fa[4];
        ldA(aA, 16 * mt, 2 * kk, CHD, lane, fa);
#pragma unroll
        for (int np = 0; np < ONT / 2; ++np) {
          uint32_t bs[4];
          ldB(aS, 16 * np, 2 * kk, CHD, lane, bs);
          mma(acc[2 * np], fa, bs[0], bs[1]);
          mma(acc[2 * np + 1], fa, bs[2], bs[3]);
        }
      }
    }
#pragma unroll
    for (int n = 0; n < ONT; ++n)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int i = 16 * mt + g_ + 8 * hh;
        const int c = 8 * n + 2 * t4;
        if (warp < 4) {                             // U = U0 - W S^T
          const float2 u0 = ld_bf16x2(stg + Q2_U0, i, c, CH64);
          const float ux = u0.x - acc[n][2 * hh], uy = u0.y - acc[n][2 * hh + 1];
          const float ds = __expf(Glast - sG[i]);
          st_bf16x2(sU, i, c, CH64, ux, uy);
          st_bf16x2(sUs, i, c, CH64, ux * ds, uy * ds);
        } else {                                    // O = e^G Q S^T (+ P U below)
          const float eg = __expf(sG[i]);
          acc[n][2 * hh] *= eg;
          acc[n][2 * hh + 1] *= eg;
        }
      }
    __syncthreads();

    // ---- state: (e^{G_last - G} U)^T K, every warp its tiles ----
    float su[SNT][4];
#pragma unroll
    for (int n = 0; n < SNT; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) su[n][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < C / 16; ++kk) {
      uint32_t fu[4];
      ldAt(aUs, 16 * kk, srl >> 3, CH64, lane, fu);
#pragma unroll
      for (int np = 0; np < SNT / 2; ++np) {
        uint32_t bk[4];
        ldBt(aK, 16 * kk, (scol >> 3) + 2 * np, CHD, lane, bk);
        mma(su[2 * np], fu, bk[0], bk[1]);
        mma(su[2 * np + 1], fu, bk[2], bk[3]);
      }
    }
    // ---- warps 4-7: O += P U, then the outputs of the slice ----
    if (warp >= 4) {
#pragma unroll
      for (int kk = 0; kk < C / 16; ++kk) {
        uint32_t fp[4];
        ldA(aP, 16 * mt, 2 * kk, CHC, lane, fp);
#pragma unroll
        for (int np = 0; np < ONT / 2; ++np) {
          uint32_t bu[4];
          ldBt(aU, 16 * kk, 2 * np, CH64, lane, bu);
          mma(acc[2 * np], fp, bu[0], bu[1]);
          mma(acc[2 * np + 1], fp, bu[2], bu[3]);
        }
      }
#pragma unroll
      for (int n = 0; n < ONT; ++n)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int i = 16 * mt + g_ + 8 * hh;
          if (i < m) {
            const int c = voff + 8 * n + 2 * t4;
            *reinterpret_cast<__nv_bfloat162*>(out + (size_t)(s0 + c0 + i) * ldo + h * D + c) =
                __floats2bfloat162_rn(scale * acc[n][2 * hh], scale * acc[n][2 * hh + 1]);
          }
        }
    }
    // ---- S <- e^{G_last} S + (e^{G_last - G} U)^T K; refresh the bf16 copy ----
    const float dl = __expf(Glast);
#pragma unroll
    for (int n = 0; n < SNT; ++n) {
      const int r0 = srl + g_, c = scol + n * 8 + 2 * t4;
#pragma unroll
      for (int e = 0; e < 4; ++e) Sr[n][e] = dl * Sr[n][e] + su[n][e];
      st_bf16x2(sS, r0, c, CHD, Sr[n][0], Sr[n][1]);
      st_bf16x2(sS, r0 + 8, c, CHD, Sr[n][2], Sr[n][3]);
    }
    __syncthreads();                                // stage j and sU / sUs / sS are free again
  }

  // ---- final state ----
#pragma unroll
  for (int n = 0; n < SNT; ++n) {
    const int r0 = srl + g_, c = scol + n * 8 + 2 * t4;
    const size_t g0 = (size_t)(voff + r0) * D + c, g8 = g0 + 8 * D;
    gS[g0] = from_f<ST>(Sr[n][0]);
    gS[g0 + 1] = from_f<ST>(Sr[n][1]);
    gS[g8] = from_f<ST>(Sr[n][2]);
    gS[g8 + 1] = from_f<ST>(Sr[n][3]);
  }
}

}  // namespace gdnc

// Chunked GDN over a varlen batch (prefill); same arguments as gdn_recurrent without the
// speculative-commit options.  dk = dv = 128.
void gdn_chunked(torch::Tensor y, torch::Tensor ba, torch::Tensor A_log, torch::Tensor dt_bias,
                 torch::Tensor state, torch::Tensor qsl, torch::Tensor slots,
                 torch::Tensor has_init, int64_t Hk, double scale, torch::Tensor out,
                 int64_t split_override) {
  const int B = slots.size(0);
  if (B == 0) return;
  const int Hv = state.size(1), DV = state.size(2), DK = state.size(3);
  TORCH_CHECK(DV == gdnc::D && DK == gdnc::D, "gdn_chunked: dk = dv = 128");
  TORCH_CHECK(A_log.scalar_type() == at::kFloat && dt_bias.scalar_type() == at::kFloat, "fp32 gates");
  TORCH_CHECK(y.stride(1) == 1 && (y.stride(0) % 8) == 0, "gdn_chunked: y rows 16-byte aligned");
  TORCH_CHECK(out.stride(1) == 1 && (out.stride(0) % 2) == 0, "gdn_chunked: out layout");
  const at::cuda::CUDAGuard guard(y.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  // value-column split: enough CTAs to cover the SMs for small batches (1, 2 or 4 per head)
  int ns = 1;
  if ((int64_t)B * Hv < 148) ns = 2;     // measured: 4-way costs more than it gains
  if (split_override > 0) ns = (int)split_override;
  TORCH_CHECK(ns == 1 || ns == 2 || ns == 4, "gdn_chunked: split 1, 2 or 4");
  dim3 grid(B, Hv, ns);
  auto run = [&](auto stag, auto ntag) {
    using ST = typename decltype(stag)::type;
    constexpr int NSc = decltype(ntag)::value;
    auto kern = gdnc::chunk_kernel<ST, NSc>;
    static bool set = false;
    if (!set) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, gdnc::SMEM));
      set = true;
    }
    C10_CUDA_CHECK(launch_pdl(kern, grid, dim3(gdnc::kThreads), gdnc::SMEM, stream,
        (const __nv_bfloat16*)y.data_ptr(), (int)y.stride(0), (const __nv_bfloat16*)ba.data_ptr(),
        (int)ba.stride(0), A_log.data_ptr<float>(), dt_bias.data_ptr<float>(),
        (ST*)state.data_ptr(), qsl.data_ptr<int>(), slots.data_ptr<int>(),
        has_init.data_ptr<int>(), (int)Hk, Hv, (float)scale, (__nv_bfloat16*)out.data_ptr(),
        (int)out.stride(0)));
  };
  struct F32 { using type = float; };
  struct BF16 { using type = __nv_bfloat16; };
  auto by_split = [&](auto stag) {
    if (ns == 1) run(stag, std::integral_constant<int, 1>{});
    else if (ns == 2) run(stag, std::integral_constant<int, 2>{});
    else run(stag, std::integral_constant<int, 4>{});
  };
  if (state.scalar_type() == at::kFloat) by_split(F32{});
  else by_split(BF16{});
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Two-phase chunked GDN (prep_kernel over every (chunk, value head), then scan_kernel over
// (sequence, value head, value slice)); same arguments as gdn_chunked plus the workspace
// (>= gdn_chunked2_ws_bytes(T, B, Hv) bytes) and the value split (2, 4 or 8; 0 = by size).
int64_t gdn_chunked2_ws_bytes(int64_t T, int64_t B, int64_t Hv) {
  return (T / gdnc::C + B) * Hv * (int64_t)gdnc::WS_CHUNK;
}

void gdn_chunked2(torch::Tensor y, torch::Tensor ba, torch::Tensor A_log, torch::Tensor dt_bias,
                  torch::Tensor state, torch::Tensor qsl, torch::Tensor slots,
                  torch::Tensor has_init, int64_t Hk, double scale, torch::Tensor out,
                  torch::Tensor ws, int64_t split_override) {
  const int B = slots.size(0);
  if (B == 0) return;
  const int T = y.size(0);
  const int Hv = state.size(1), DV = state.size(2), DK = state.size(3);
  TORCH_CHECK(DV == gdnc::D && DK == gdnc::D, "gdn_chunked2: dk = dv = 128");
  TORCH_CHECK(A_log.scalar_type() == at::kFloat && dt_bias.scalar_type() == at::kFloat, "fp32 gates");
  TORCH_CHECK(y.stride(1) == 1 && (y.stride(0) % 8) == 0 &&
                  (reinterpret_cast<uintptr_t>(y.data_ptr()) % 16) == 0,
              "gdn_chunked2: y rows 16-byte aligned");
  TORCH_CHECK(out.stride(1) == 1 && (out.stride(0) % 2) == 0, "gdn_chunked2: out layout");
  TORCH_CHECK(ws.is_cuda() && ws.numel() * ws.element_size() >= gdn_chunked2_ws_bytes(T, B, Hv) &&
                  (reinterpret_cast<uintptr_t>(ws.data_ptr()) % 16) == 0, "gdn_chunked2: workspace");
  const at::cuda::CUDAGuard guard(y.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  // phase 1: every chunk of the flattened batch (an upper bound; CTAs past the end return)
  const int max_chunks = T / gdnc::C + B;
  {
    static bool set = false;
    if (!set) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(gdnc::prep_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, gdnc::SMEM1));
      set = true;
    }
    C10_CUDA_CHECK(launch_pdl(gdnc::prep_kernel, dim3(max_chunks, Hv), dim3(gdnc::kThreads),
                              gdnc::SMEM1, stream, (const __nv_bfloat16*)y.data_ptr(),
                              (int)y.stride(0), (const __nv_bfloat16*)ba.data_ptr(),
                              (int)ba.stride(0), A_log.data_ptr<float>(), dt_bias.data_ptr<float>(),
                              qsl.data_ptr<int>(), B, (int)Hk, Hv, (uint8_t*)ws.data_ptr()));
  }
  // phase 2: split the value columns until the grid covers the SMs
  int ns = 2;
  while (ns < 8 && (int64_t)B * Hv * ns < 148) ns *= 2;
  if (split_override > 0) ns = (int)split_override;
  TORCH_CHECK(ns == 2 || ns == 4 || ns == 8, "gdn_chunked2: split 2, 4 or 8");
  dim3 grid(B, Hv, ns);
  auto run = [&](auto stag, auto ntag) {
    using ST = typename decltype(stag)::type;
    constexpr int NSc = decltype(ntag)::value;
    auto kern = gdnc::scan_kernel<ST, NSc>;
    static bool set = false;
    if (!set) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, gdnc::SMEM2));
      set = true;
    }
    C10_CUDA_CHECK(launch_pdl(kern, grid, dim3(gdnc::kThreads), gdnc::SMEM2, stream,
        (const __nv_bfloat16*)y.data_ptr(), (int)y.stride(0), (ST*)state.data_ptr(),
        qsl.data_ptr<int>(), slots.data_ptr<int>(), has_init.data_ptr<int>(), (int)Hk, Hv,
        (float)scale, (const uint8_t*)ws.data_ptr(), (__nv_bfloat16*)out.data_ptr(),
        (int)out.stride(0)));
  };
  struct F32 { using type = float; };
  struct BF16 { using type = __nv_bfloat16; };
  auto by_split = [&](auto stag) {
    if (ns == 2) run(stag, std::integral_constant<int, 2>{});
    else if (ns == 4) run(stag, std::integral_constant<int, 4>{});
    else run(stag, std::integral_constant<int, 8>{});
  };
  if (state.scalar_type() == at::kFloat) by_split(F32{});
  else by_split(BF16{});
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace rad
