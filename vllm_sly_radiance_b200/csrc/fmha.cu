// Chunked-prefill attention on 5th-generation tensor cores: paged fp8 (e4m3) KV cache, head
// dim 256, grouped-query heads packed into the query rows, causal.
//
// Reference behaviour: the libr4d prefill kernel r4d_attn_prefill_h256_gqa6 with its fp8 QK and
// PV legs, double-buffered K/V staging and heaviest-q-block-first dispatch
// (sly/r4d/r4d_extras_rx10.patch:393-510 O_QK8 / O_PV8 / O_DB / O_HVF, radiance_r4d_hybrid_attn.py:378).
//
// B200 design (one CTA per 128 query rows of one kv head):
//  * Rows are (token, q head of the group) pairs, the packing the other attention kernels use, so
//    the six heads of a group share every K/V tile.  Q is gathered once, rounded to e4m3 (it is
//    e4m3-valued already when the cache is fp8) and stored as two 128-byte-swizzled halves.
//  * S = Q K^T: tcgen05.mma.kind::f8f6f4 (e4m3 x e4m3, fp32 accumulate), M = 128 rows, N = 128
//    keys, eight K = 32 steps, into one of two TMEM S buffers, so the next tile's S is computed
//    while the softmax of this one runs.
//  * Softmax: four warps, one row per thread (the TMEM lane), online max / sum in the exp2
//    domain; P = 256 * exp2(s - m) as e4m3 into shared memory (the scale keeps small
//    probabilities out of the subnormal range; O is divided by 256 l at the end).  O is rescaled
//    in TMEM only when a warp's running maximum moved.
//  * O += P V: tcgen05.mma.kind::f8f6f4 with V as an MN-major operand straight from the paged
//    cache layout (keys x dims), M = 128, N = 256, O (256 fp32 columns) stays in TMEM for the
//    whole key range.
//  * K and V pages arrive by TMA (two 64-key pages x two 128-byte halves per 128-key tile) into a
//    two-stage ring; all waits are bounded (status word).
//  * Causal tiles are scheduled heaviest first: CTA x takes row tile (last - x).
// Warp roles (320 threads): warps 0-7 softmax + epilogue (two threads per query row), warp 8 TMA
// producer, warp 9 MMA issuer.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <array>
#include <map>

#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "tma_host.h"

namespace rad {
namespace fmha {

constexpr int D = 256;
constexpr int BM = 128;                 // query rows per CTA
constexpr int BN = 128;                 // keys per tile
constexpr int PAGE = 64;                // KV page rows (TMA box)
constexpr int HALF = BM * 128;          // one 128-byte column half of a 128-row tile: 16 KB
constexpr int Q_BYTES = 2 * HALF;
constexpr int KV_BYTES = 2 * HALF;
constexpr int P_BYTES = BM * BN;
constexpr int STAGES = 2;
constexpr int kSoftThreads = 256;      // softmax / epilogue warps 0-7
constexpr int kTmaWarp = 8, kMmaWarp = 9;
constexpr int kThreads = kSoftThreads + 64;
constexpr int P_BUFS = 2;              // P tiles: softmax(j) writes one while PV(j - 1) reads the other
constexpr int SMEM_BYTES = 1024 + Q_BYTES + STAGES * 2 * KV_BYTES + P_BUFS * P_BYTES + 4096;   // + barriers
// The running row maximum is raised (and O rescaled) only when a tile's maximum exceeds it by more
// than this many log2 units; P = 2^(s - m + 8) then stays below 2^8.75 = 430 < 448 (e4m3 max).
constexpr float kRescaleLog2 = 0.75f;
constexpr uint32_t O_COL = 0, S_COL = 256;      // TMEM: O [0, 256), S buffers [256, 384), [384, 512)

// kind::f8f6f4 instruction descriptor: e4m3 x e4m3 -> fp32, M = 128
__host__ __device__ constexpr uint32_t idesc_f8(int n, bool b_mn_major) {
  return (1u << 4)                              // D format F32
         | (0u << 7) | (0u << 10)               // A, B format E4M3
         | ((b_mn_major ? 1u : 0u) << 16)       // B major-ness
         | ((uint32_t)(n >> 3) << 17)
         | ((uint32_t)(BM >> 4) << 24);
}

// MN-major 128-byte-swizzled operand: rows of 128 bytes along MN, 8-row atoms along K 1024 bytes
// apart (SBO), 128-byte MN blocks `lbo` bytes apart (LBO)
DEVI uint64_t sdesc_sw128_mn(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

DEVI void tmem_ld_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
DEVI void tmem_st_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// 2^x on the multi-function unit (PTX ex2.approx.ftz: relative error ~2^-22, -inf -> +0); the
// probabilities it feeds are rounded to e4m3 next, so its error is far below theirs
DEVI float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Softmax arithmetic on the sm_100 paired / three-input forms: one instruction per two scores
// for the scale-and-shift and the running sums, one per two for the row maximum.
DEVI float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
DEVI float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
DEVI float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// two non-negative, finite P values -> e4m3 pair, lo in the low byte (saturating at 448)
DEVI uint32_t p_to_e4m3x2(float lo, float hi) {
  uint16_t d;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(d) : "f"(hi), "f"(lo));
  return d;
}

struct Bars {
  uint64_t q_full;
  uint64_t k_full[STAGES], v_full[STAGES], kv_empty[STAGES];
  uint64_t s_full[2], s_empty[2];
  uint64_t p_full[P_BUFS], pv_done[P_BUFS];
  float row_max[2][2][BM];      // [S buffer][half][row]: the halves' partial row maxima
  float row_sum[2][BM];         // [half][row]: the halves' final sums
  uint32_t tmem_slot;
  int abort;
};
static_assert(sizeof(Bars) <= 4096, "barrier block");

__global__ void __launch_bounds__(kThreads, 1) fmha_prefill_kernel(
    const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
    const __nv_bfloat16* __restrict__ q, const int* __restrict__ block_tables, int bt_stride,
    const int* __restrict__ seq_lens, const int* __restrict__ qsl, const int* __restrict__ tile_seq,
    const int* __restrict__ tile_row0, int num_tiles, int Hq, int Hkv, float scale_log2,
    __nv_bfloat16* __restrict__ out, int* __restrict__ status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + Q_BYTES;                       // stage s: K at s * 2 * KV_BYTES, V after it
  uint8_t* sP = sKV + STAGES * 2 * KV_BYTES;
  Bars* bar = reinterpret_cast<Bars*>(sP + P_BUFS * P_BYTES);

  pdl_wait();     // q (prologue) and the cache writes precede this kernel
  pdl_trigger();
  // heaviest first: the last row tile of a sequence has the longest causal key range
  const int tile = num_tiles - 1 - blockIdx.x;
  const int hk = blockIdx.y;
  const int row0 = tile_row0[tile];
  if (row0 % BM != 0) return;          // the metadata lists 64-row tiles: take every other one
  const int b = tile_seq[tile];
  const int G = Hq / Hkv;
  const int s0 = qsl[b];
  const int ql = qsl[b + 1] - s0;
  const int L = seq_lens[b];
  const int R = ql * G;
  const int rows_here = min(BM, R - row0);
  const int last_i = (row0 + rows_here - 1) / G;
  const int kv_end = L - ql + last_i + 1;            // causal: keys up to the last row's position
  const int nt = (kv_end + BN - 1) / BN;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    mbar_init(&bar->q_full, kSoftThreads);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bar->k_full[s], 1);
      mbar_init(&bar->v_full[s], 1);
      mbar_init(&bar->kv_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar->s_full[s], 1);
      mbar_init(&bar->s_empty[s], kSoftThreads);
    }
    for (int s = 0; s < P_BUFS; ++s) {
      mbar_init(&bar->p_full[s], kSoftThreads);
      mbar_init(&bar->pv_done[s], 1);
    }
    bar->abort = 0;
    fence_mbar_init();
  }
  if (warp == kTmaWarp && lane == 0) {
    tma_prefetch_desc(&tmap_k);
    tma_prefetch_desc(&tmap_v);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&bar->tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_slot;

  if (warp == kTmaWarp) {
    // ---------------- TMA producer: K and V pages of each 128-key tile ----------------
    if (elect_one()) {
      const int* bt = block_tables + (size_t)b * bt_stride;
      for (int j = 0; j < nt; ++j) {
        const int s = j % STAGES;
        if (j >= STAGES && !mbar_wait(&bar->kv_empty[s], ((j / STAGES) - 1) & 1, status)) {
          bar->abort = 1;
          break;
        }
        const int key0 = j * BN;
        const int pg0 = bt[key0 / PAGE];
        const int pg1 = key0 + PAGE < kv_end ? bt[key0 / PAGE + 1] : pg0;   // past the range: any
        uint8_t* sk = sKV + s * 2 * KV_BYTES;                             // valid (finite) page
        uint8_t* sv = sk + KV_BYTES;
        mbar_arrive_expect_tx(&bar->k_full[s], KV_BYTES);
        mbar_arrive_expect_tx(&bar->v_full[s], KV_BYTES);
        const int pgs[2] = {pg0, pg1};
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const int row = (pgs[p] * Hkv + hk) * PAGE;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            tma_load_2d(sk + h * HALF + p * PAGE * 128, &tmap_k, &bar->k_full[s], h * 128, row);
            tma_load_2d(sv + h * HALF + p * PAGE * 128, &tmap_v, &bar->v_full[s], h * 128, row);
          }
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (elect_one()) {
      bool ok = mbar_wait(&bar->q_full, 0, status);
      tc_fence_after();
      const uint32_t qa = smem_u32(sQ);
      const uint32_t idesc_s = idesc_f8(BN, false);
      const uint32_t idesc_o = idesc_f8(D, true);
      auto issue_s = [&](int j) -> bool {
        const int s = j % STAGES, sb = j & 1;
        if (!mbar_wait(&bar->k_full[s], (j / STAGES) & 1, status)) return false;
        if (j >= 2 && !mbar_wait(&bar->s_empty[sb], ((j >> 1) - 1) & 1, status)) return false;
        tc_fence_after();
        const uint32_t ka = smem_u32(sKV + s * 2 * KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 32; ++kk) {
          const uint32_t off = (kk / 4) * HALF + (kk % 4) * 32;
          mma_f8(tmem + S_COL + sb * BN, sdesc_sw128(qa + off), sdesc_sw128(ka + off), idesc_s,
                 kk > 0 ? 1u : 0u);
        }
        mma_commit(&bar->s_full[sb]);
        return true;
      };
      if (ok && nt > 0) ok = issue_s(0);
      for (int j = 0; j < nt && ok; ++j) {
        if (j + 1 < nt && !issue_s(j + 1)) { ok = false; break; }
        const int s = j % STAGES, pb = j & 1;
        if (!mbar_wait(&bar->p_full[pb], (j >> 1) & 1, status) ||
            !mbar_wait(&bar->v_full[s], (j / STAGES) & 1, status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t pa = smem_u32(sP + pb * P_BYTES);
        const uint32_t va = smem_u32(sKV + s * 2 * KV_BYTES + KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < BN / 32; ++kk)
          mma_f8(tmem + O_COL, sdesc_sw128(pa + kk * 32), sdesc_sw128_mn(va + kk * 32 * 128, HALF),
                 idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&bar->pv_done[pb]);
        mma_commit(&bar->kv_empty[s]);
      }
      if (!ok) bar->abort = 1;
    }
  } else {
    // ---------------- softmax + epilogue: two threads per query row ----------------
    // warp w owns TMEM lanes 32 (w % 4) .. + 31 (the rows); half hf = w / 4 takes key columns
    // [64 hf, 64 hf + 64) of each S tile and O columns [128 hf, 128 hf + 128).  The halves swap
    // their row maxima through shared memory once per tile; each keeps its own running sum.
    const int hf = warp >> 2;
    const int r = (warp & 3) * 32 + lane;              // row within the tile
    const int rr = row0 + r;
    const bool valid = rr < R;
    const int i = valid ? rr / G : 0;
    const int head = hk * G + (valid ? rr % G : 0);
    const int pos = L - ql + i;
    // Q row -> e4m3, this half's 128-byte half of the two swizzled halves
    {
      const __nv_bfloat16* src = q + ((size_t)(s0 + i) * Hq + head) * D;
#pragma unroll 4
      for (int c = hf * 8; c < hf * 8 + 8; ++c) {
        uint4 w = make_uint4(0, 0, 0, 0);
        if (valid) {
          const uint4 u0 = reinterpret_cast<const uint4*>(src)[2 * c];
          const uint4 u1 = reinterpret_cast<const uint4*>(src)[2 * c + 1];
          const __nv_bfloat162* h0 = reinterpret_cast<const __nv_bfloat162*>(&u0);
          const __nv_bfloat162* h1 = reinterpret_cast<const __nv_bfloat162*>(&u1);
          uint16_t pk[8];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 a = __bfloat1622float2(h0[e]), bb = __bfloat1622float2(h1[e]);
            pk[e] = f32x2_to_e4m3x2(a.x, a.y);
            pk[4 + e] = f32x2_to_e4m3x2(bb.x, bb.y);
          }
          w = *reinterpret_cast<uint4*>(pk);
        }
        const int h = c / 8, ch = c % 8;
        *reinterpret_cast<uint4*>(sQ + h * HALF + r * 128 + ((ch ^ (r & 7)) * 16)) = w;
      }
    }
    fence_proxy_async();
    mbar_arrive(&bar->q_full);

    constexpr int HC = BN / 2;                         // key columns per half
    static_assert(HC == 64, "softmax half-tile of 64 keys");
    // l_run: this half's share of the row sum of 256 p (the e4m3 P operand's scale)
    float m_run = -INFINITY, l_run = 0.f;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const float2 sc2 = make_float2(scale_log2, scale_log2);
    // Every softmax thread runs all nt iterations and reaches each named barrier: a failed wait
    // only turns the rest of the work off (ok is warp-uniform), so no barrier is left short.
    bool ok = true;
    for (int j = 0; j < nt; ++j) {
      const int sb = j & 1;
      if (ok) ok = mbar_wait(&bar->s_full[sb], (j >> 1) & 1, status);
      ok = __all_sync(0xffffffffu, ok);
      const int kbase = j * BN + hf * HC;
      // keys [kbase, kbase + 64) all live for every valid row of the warp: no causal mask
      const bool unmasked =
          __all_sync(0xffffffffu, !valid || (kbase + HC - 1 <= pos && kbase + HC <= L));
      float sv[HC];
      if (ok) {
        tc_fence_after();
        uint32_t u0[32], u1[32];
        tmem_ld_x32(tmem + lane_base + S_COL + sb * BN + hf * HC, u0);
        tmem_ld_x32(tmem + lane_base + S_COL + sb * BN + hf * HC + 32, u1);
        tmem_ld_wait();
        if (unmasked) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            sv[e] = __uint_as_float(u0[e]);
            sv[32 + e] = __uint_as_float(u1[e]);
          }
        } else {
          // live keys: key <= pos and key < L, i.e. e < lim within this half-tile
          const int lim = valid ? min(pos + 1, L) - kbase : 0;
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            sv[e] = e < lim ? __uint_as_float(u0[e]) : -INFINITY;
            sv[32 + e] = e + 32 < lim ? __uint_as_float(u1[e]) : -INFINITY;
          }
        }
        tc_fence_before();
        mbar_arrive(&bar->s_empty[sb]);             // S buffer free for tile j + 2
      } else {
#pragma unroll
        for (int e = 0; e < HC; ++e) sv[e] = -INFINITY;
      }
      float mx8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float t = fmax3(sv[k], sv[k + 8], sv[k + 16]);
        t = fmax3(t, sv[k + 24], sv[k + 32]);
        t = fmax3(t, sv[k + 40], sv[k + 48]);
        mx8[k] = fmaxf(t, sv[k + 56]);
      }
      float mx = fmax3(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], mx8[5]),
                       fmaxf(mx8[6], mx8[7]));
      bar->row_max[sb][hf][r] = mx;
      asm volatile("bar.sync 1, %0;" ::"n"(kSoftThreads) : "memory");
      mx = fmaxf(mx, bar->row_max[sb][hf ^ 1][r]);
      // scale > 0: the max commutes with it.  The running maximum moves only when the tile's
      // exceeds it by more than kRescaleLog2 (both halves of a row decide alike: same inputs).
      const float mx_s = mx * scale_log2;
      const bool grow = mx_s > m_run + kRescaleLog2;       // m_run = -inf: any finite maximum
      const float m_new = grow ? mx_s : m_run;
      const float mref = m_new == -INFINITY ? 0.f : m_new;
      const bool need = grow && m_run != -INFINITY;        // O holds terms at the old maximum
      const float alpha = need ? ex2_approx(m_run - m_new) : (grow ? 0.f : 1.f);
      // 256 p = 2^(s * scale_log2 - mref + 8): the x256 of the e4m3 P operand rides in the
      // exponent; masked scores give ex2(-inf) = 0.  P goes to e4m3 as it is made.
      const float2 off2 = make_float2(8.f - mref, 8.f - mref);
      float2 acc0 = make_float2(0.f, 0.f), acc1 = acc0, acc2 = acc0, acc3 = acc0;
      uint32_t pw[HC / 4];
#pragma unroll
      for (int e = 0; e < HC; e += 8) {
        const float2 x0 = ffma2(make_float2(sv[e], sv[e + 1]), sc2, off2);
        const float2 x1 = ffma2(make_float2(sv[e + 2], sv[e + 3]), sc2, off2);
        const float2 x2 = ffma2(make_float2(sv[e + 4], sv[e + 5]), sc2, off2);
        const float2 x3 = ffma2(make_float2(sv[e + 6], sv[e + 7]), sc2, off2);
        const float2 p0 = make_float2(ex2_approx(x0.x), ex2_approx(x0.y));
        const float2 p1 = make_float2(ex2_approx(x1.x), ex2_approx(x1.y));
        const float2 p2 = make_float2(ex2_approx(x2.x), ex2_approx(x2.y));
        const float2 p3 = make_float2(ex2_approx(x3.x), ex2_approx(x3.y));
        acc0 = fadd2(acc0, p0);
        acc1 = fadd2(acc1, p1);
        acc2 = fadd2(acc2, p2);
        acc3 = fadd2(acc3, p3);
        pw[e / 4] = p_to_e4m3x2(p0.x, p0.y) | (p_to_e4m3x2(p1.x, p1.y) << 16);
        pw[e / 4 + 1] = p_to_e4m3x2(p2.x, p2.y) | (p_to_e4m3x2(p3.x, p3.y) << 16);
      }
      const float2 accs = fadd2(fadd2(acc0, acc1), fadd2(acc2, acc3));
      l_run = l_run * alpha + (accs.x + accs.y);
      m_run = m_new;
      // O may be rescaled once PV(j - 1) is done; P buffer pb is free once PV(j - 2) is done
      // (implied by PV(j - 1): the MMAs complete in issue order)
      const int pb = j & 1;
      const bool resc = __any_sync(0xffffffffu, need) && j > 0;
      if (ok && resc) ok = mbar_wait(&bar->pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, status);
      else if (ok && j >= 2) ok = mbar_wait(&bar->pv_done[pb], ((j >> 1) - 1) & 1, status);
      ok = __all_sync(0xffffffffu, ok);
      if (ok && resc) {
        tc_fence_after();
        {
          const float a_o = need ? alpha : 1.f;
          for (int c = 0; c < D / 64; ++c) {
            uint32_t u[32];
            const uint32_t col = O_COL + hf * (D / 2) + c * 32;
            tmem_ld_x32(tmem + lane_base + col, u);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) u[e] = __float_as_uint(__uint_as_float(u[e]) * a_o);
            tmem_st_x32(tmem + lane_base + col, u);
          }
          tmem_st_wait();
        }
      }
      if (!ok) continue;                             // no barrier below: safe to skip
      // this half's 64 e4m3 columns of row r of the swizzled P tile
#pragma unroll
      for (int c = 0; c < HC / 16; ++c) {
        const int cc = hf * (HC / 16) + c;
        *reinterpret_cast<uint4*>(sP + pb * P_BYTES + r * 128 + ((cc ^ (r & 7)) * 16)) =
            make_uint4(pw[4 * c], pw[4 * c + 1], pw[4 * c + 2], pw[4 * c + 3]);
      }
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(&bar->p_full[pb]);
    }
    // ---- epilogue: O / l -> bf16, l = the two halves' sums of 256 p ----
    bar->row_sum[hf][r] = l_run;
    asm volatile("bar.sync 1, %0;" ::"n"(kSoftThreads) : "memory");
    const float l_tot = l_run + bar->row_sum[hf ^ 1][r];
    if (ok && nt > 0) ok = mbar_wait(&bar->pv_done[(nt - 1) & 1], ((nt - 1) >> 1) & 1, status);
    tc_fence_after();
    const float inv = (ok && l_tot > 0.f) ? 1.f / l_tot : 0.f;      // l_tot sums 256 p
    __nv_bfloat16* dst = out + ((size_t)(s0 + i) * Hq + head) * D + hf * (D / 2);
    for (int c = 0; c < D / 64; ++c) {
      uint32_t u[32];
      tmem_ld_x32(tmem + lane_base + O_COL + hf * (D / 2) + c * 32, u);
      tmem_ld_wait();
      if (valid) {
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const __nv_bfloat162 hh = __floats2bfloat162_rn(__uint_as_float(u[2 * e]) * inv,
                                                          __uint_as_float(u[2 * e + 1]) * inv);
          w[e] = *reinterpret_cast<const uint32_t*>(&hh);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e)
          reinterpret_cast<uint4*>(dst + c * 32)[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}


// ---------------------------------------------------------------------------------------------
// int4 (KV4) pages -> e4m3 pages for the prefill kernel.  A 4-bit cache row is D/2 code bytes
// (low nibble = even element) and one fp16 (scale, zero) pair per 16 elements: v = code * scale
// + zero.  Before a prefill chunk attends over such a cache, every key its sequences reach is
// dequantised once into a compact e4m3 copy in 64-key pages (the TMA box of the prefill kernel;
// the 4-bit cache may use smaller pages), pages renumbered per sequence, and the tcgen05 kernel
// runs on that copy.  The copy costs one read of the 4-bit rows and one e4m3 write per chunk and
// layer -- small next to the chunk's attention over the same keys.
// grid (64-key pages of the table, sequences, kv heads); a thread converts 16-element groups.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) kv4_to_e4m3_pages_kernel(
    const uint8_t* __restrict__ k4, const uint8_t* __restrict__ v4,
    const int* __restrict__ block_tables, int bt_stride, int nb, int block_size,
    const int* __restrict__ seq_lens, int Hkv, uint8_t* __restrict__ k8, uint8_t* __restrict__ v8,
    int* __restrict__ bt_out, int bt_out_stride) {
  pdl_wait();     // the chunk's keys were written by the preceding prologue
  pdl_trigger();
  constexpr int RB = D / 2 + D / 4;              // 4-bit row bytes (codes + fp16 pairs)
  constexpr int G = D / 16;                      // 16-element groups per row
  const int p = blockIdx.x, b = blockIdx.y, hk = blockIdx.z;
  const int len = seq_lens[b], pages = (len + PAGE - 1) / PAGE;
  if (p >= pages || p * PAGE >= nb * block_size) return;
  int dst = p;
  for (int i = 0; i < b; ++i) dst += (seq_lens[i] + PAGE - 1) / PAGE;
  if (hk == 0 && threadIdx.x == 0) bt_out[(size_t)b * bt_out_stride + p] = dst;
  const size_t d_off = ((size_t)dst * Hkv + hk) * PAGE * D;
  const int last_key = min(len, nb * block_size) - 1;
  for (int idx = threadIdx.x; idx < 2 * PAGE * G; idx += blockDim.x) {
    const int which = idx / (PAGE * G), rem = idx % (PAGE * G);
    const int r = rem / G, g = rem % G;
    // rows past the sequence repeat its last key (masked; their table slots may be unset)
    const int key = min(p * PAGE + r, last_key);
    const int blk = block_tables[(size_t)b * bt_stride + key / block_size];
    const uint8_t* row = (which ? v4 : k4) +
                         (((size_t)blk * Hkv + hk) * block_size + key % block_size) * RB;
    const uint2 codes = *reinterpret_cast<const uint2*>(row + g * 8);
    const __half2 sz = *reinterpret_cast<const __half2*>(row + D / 2 + g * 4);
    const float sc = __low2float(sz), zr = __high2float(sz);
    uint16_t o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t word = e < 4 ? codes.x : codes.y;
      const int sh = (e % 4) * 8;
      o[e] = f32x2_to_e4m3x2((float)((word >> sh) & 0xF) * sc + zr,
                             (float)((word >> (sh + 4)) & 0xF) * sc + zr);
    }
    *reinterpret_cast<uint4*>((which ? v8 : k8) + d_off + (size_t)r * D + g * 16) =
        *reinterpret_cast<const uint4*>(o);
  }
}

}  // namespace fmha

static std::mutex g_fmha_mu;
// keyed by the cache's address and every dimension: a cache freed and another allocated at the
// same address with another shape (an engine rebuilt with other TP or pool sizes) gets its own map
static std::map<std::array<int64_t, 5>, CUtensorMap> g_fmha_maps;

static CUtensorMap cache_map(const torch::Tensor& cache) {
  std::lock_guard<std::mutex> lk(g_fmha_mu);
  const std::array<int64_t, 5> key{(int64_t)reinterpret_cast<uintptr_t>(cache.data_ptr()),
                                   cache.size(0), cache.size(1), cache.size(2), cache.size(3)};
  auto it = g_fmha_maps.find(key);
  if (it != g_fmha_maps.end()) return it->second;
  const int64_t rows = cache.size(0) * cache.size(1) * cache.size(2);
  CUtensorMap m = make_tma_2d(cache.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, fmha::D, rows,
                              fmha::D, 128, fmha::PAGE, CU_TENSOR_MAP_SWIZZLE_128B);
  g_fmha_maps.emplace(key, m);
  return m;
}

// Causal prefill attention over an e4m3 paged cache [blocks, Hkv, 64, 256]: q [T, Hq, 256] bf16
// (e4m3-valued), tiles listed in 64-row steps as for paged_attention (the kernel takes the
// 128-row-aligned ones), out [T, Hq, 256] bf16.
void fmha_prefill(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                  torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor qsl,
                  torch::Tensor tile_seq, torch::Tensor tile_row0, double scale, torch::Tensor out,
                  torch::Tensor status) {
  using namespace fmha;
  const int T = q.size(0), Hq = q.size(1);
  const int Hkv = k_cache.size(1);
  const int num_tiles = tile_seq.size(0);
  if (T == 0 || num_tiles == 0) return;
  TORCH_CHECK(q.size(2) == D && q.is_contiguous() && q.scalar_type() == at::kBFloat16, "fmha: q");
  TORCH_CHECK(k_cache.scalar_type() == at::kFloat8_e4m3fn && v_cache.scalar_type() == at::kFloat8_e4m3fn &&
                  k_cache.size(2) == PAGE && k_cache.size(3) == D && k_cache.is_contiguous() &&
                  v_cache.is_contiguous(), "fmha: e4m3 cache [blocks, Hkv, 64, 256]");
  TORCH_CHECK(Hq % Hkv == 0, "fmha: grouped heads");
  TORCH_CHECK(out.is_contiguous() && out.scalar_type() == at::kBFloat16, "fmha: out");
  const at::cuda::CUDAGuard guard(q.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  CUtensorMap tk = cache_map(k_cache), tv = cache_map(v_cache);
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(fmha_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        SMEM_BYTES));
    attr = true;
  }
  int* st = status.numel() ? status.data_ptr<int>() : nullptr;
  C10_CUDA_CHECK(launch_pdl(fmha_prefill_kernel, dim3(num_tiles, Hkv), dim3(kThreads), SMEM_BYTES,
                            stream, tk, tv, (const __nv_bfloat16*)q.data_ptr(),
                            block_tables.data_ptr<int>(), (int)block_tables.stride(0),
                            seq_lens.data_ptr<int>(), qsl.data_ptr<int>(), tile_seq.data_ptr<int>(),
                            tile_row0.data_ptr<int>(), num_tiles, Hq, Hkv,
                            (float)(scale * 1.4426950408889634), (__nv_bfloat16*)out.data_ptr(), st));
}

// int4 caches [blocks, Hkv, block_size, D/2 + D/4] -> compact e4m3 pages k8 / v8 [>= sum of
// 64-key pages, Hkv, 64, D] for the sequences of the batch, with their 64-key block table in
// bt_out [B, ceil(table width * block_size / 64)].
void kv4_to_e4m3_pages(torch::Tensor k4, torch::Tensor v4, torch::Tensor block_tables,
                       torch::Tensor seq_lens, torch::Tensor k8, torch::Tensor v8,
                       torch::Tensor bt_out) {
  using namespace fmha;
  const int B = block_tables.size(0), nb = block_tables.size(1), Hkv = k4.size(1);
  const int bs = k4.size(2);
  TORCH_CHECK(k4.scalar_type() == at::kByte && v4.scalar_type() == at::kByte && k4.dim() == 4 &&
                  k4.size(3) == D / 2 + D / 4 && k4.is_contiguous() && v4.is_contiguous() && bs >= 1,
              "kv4_to_e4m3_pages: 4-bit cache [blocks, Hkv, block_size, 192]");
  const int p64 = (nb * bs + PAGE - 1) / PAGE;
  TORCH_CHECK(k8.scalar_type() == at::kFloat8_e4m3fn && v8.scalar_type() == at::kFloat8_e4m3fn &&
                  k8.size(1) == Hkv && k8.size(2) == PAGE && k8.size(3) == D && k8.is_contiguous() &&
                  v8.is_contiguous() && k8.size(0) >= (int64_t)B * p64, "kv4_to_e4m3_pages: e4m3 pages");
  TORCH_CHECK(bt_out.dim() == 2 && bt_out.size(0) == B && bt_out.size(1) >= p64 &&
                  bt_out.stride(1) == 1 && bt_out.scalar_type() == at::kInt,
              "kv4_to_e4m3_pages: 64-key block table");
  TORCH_CHECK(block_tables.stride(1) == 1 && block_tables.scalar_type() == at::kInt,
              "kv4_to_e4m3_pages: block table rows");
  if (B == 0 || nb == 0) return;
  const at::cuda::CUDAGuard guard(k4.device());
  C10_CUDA_CHECK(launch_pdl(kv4_to_e4m3_pages_kernel, dim3(p64, B, Hkv), dim3(256), 0,
                            at::cuda::getCurrentCUDAStream(), (const uint8_t*)k4.data_ptr(),
                            (const uint8_t*)v4.data_ptr(), block_tables.data_ptr<int>(),
                            (int)block_tables.stride(0), nb, bs, seq_lens.data_ptr<int>(), Hkv,
                            (uint8_t*)k8.data_ptr(), (uint8_t*)v8.data_ptr(),
                            bt_out.data_ptr<int>(), (int)bt_out.stride(0)));
}

}  // namespace rad
