// MX-format W4A8 / W6A8 / W8A8 linear on 5th-generation tensor cores (sm_100a).
//
//   C[m, n] = a_scale[m] * sum_k e4m3(A[m, k]) * w(W[n, k]) * 2^(ws[n, k/32] - 127)
//
// w is the weight element type, picked per call from the stored row width: e2m1 (MXFP4, K/2
// bytes a row), e2m3 (MXFP6, 3K/4 bytes) or e4m3 (MXFP8, K bytes).  All three are native to
// kind::mxf8f6f4; only the TMA map type, the transaction bytes and the MMA's A-format field change.
//
// Reference behaviour: the W4A8 GEMM family of sly/mxfp4/radiance_mxfp4_fp8.hip (:132 per-block,
// :327 folded, :666 A-tiled prefill, :983 split-K decode).  The B200 design is different:
//
//  * One tcgen05.mma.kind::mxf8f6f4.block_scale instruction does the e2m1 x e4m3 product with the
//    per-32 UE8M0 weight scales applied inside the tensor core (no folded/PSW weight repack).
//  * Weights are the MMA "A" operand (M_mma = 128 weight rows) and activations the "B" operand
//    (N_mma = BN tokens, 16..256).  The same kernel serves decode (BN = 16, tokens padded by TMA
//    zero-fill) and prefill (BN = 256): the swap-AB orientation the reference emulates with its
//    separate decode kernel.
//  * Weight tiles arrive by TMA with the 16U4_ALIGN16B map type, which expands packed nibbles to
//    the padded form the f8f6f4 MMA reads; scale factors arrive by one 512-byte bulk copy per
//    128x128 tile and go to tensor memory with tcgen05.cp.  Activation scale factors are a
//    constant 1.0 in tensor memory: activations carry a per-token fp32 scale applied in the
//    epilogue (the reference's per-token e4m3 contract).
//  * Split-K for small M runs as a thread-block cluster along K: each CTA accumulates its K range
//    in its own TMEM, the partial tiles are reduced through distributed shared memory, and the
//    cluster writes the output once.  This replaces the reference's global fp32 partials and
//    self-resetting counter (radiance_mxfp4_fp8.hip:1251-1343) with no global workspace.
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM allocator + MMA issuer,
// warps 2..5 = epilogue (their warp-in-quad index covers the four TMEM lane quarters).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "finish.cuh"
#include "tma_host.h"

namespace rad {
namespace mxfp4 {

constexpr int BM = 128;          // weight rows per tile (MMA M)
constexpr int BK = 128;          // K elements per pipeline stage (4 MMAs of K = 32)
constexpr int W_TILE_BYTES = BM * BK;          // padded e2m1: 1 byte per element in smem
// weight element types: code 0 = e2m1 (16U4_ALIGN16B), 1 = e2m3 (16U6_ALIGN16B), 2 = e4m3 (UINT8).
// TMA transaction bytes are the packed source bytes; the shared-memory tile is one byte per
// element for all three (16 codes in a 16-byte group, the form the f8f6f4 MMA reads).
__host__ __device__ constexpr uint32_t w_tile_tx(int wfmt) {
  return wfmt == 0 ? BM * BK / 2 : wfmt == 1 ? BM * BK * 3 / 4 : BM * BK;
}
__host__ __device__ constexpr uint32_t w_mma_format(int wfmt) {
  return wfmt == 0 ? 5u : wfmt == 1 ? 3u : 0u;          // E2M1 / E2M3 / E4M3
}
constexpr int SF_TILE_BYTES = 512;
constexpr int kThreads = 192;
constexpr int kSmemBudget = 227 * 1024;

template <int BN>
struct Cfg {
  static constexpr int A_TILE_BYTES = BN * BK;
  // stages start on 1024-byte boundaries (128B-swizzled tiles need it)
  static constexpr int STAGE_BYTES = (W_TILE_BYTES + A_TILE_BYTES + SF_TILE_BYTES + 1023) / 1024 * 1024;
  // decode tiles (BN <= 64) keep two CTAs per SM so a split-K grid runs in a single wave;
  // prefill tiles take the whole SM
  static constexpr int MIN_BLOCKS = BN <= 64 ? 2 : 1;
  static constexpr int BUDGET = MIN_BLOCKS == 2 ? (228 * 1024 / 2 - 1024 - 3072) : (kSmemBudget - 2048);
  static constexpr int STAGES_RAW = BUDGET / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  // TMEM columns: accumulator BN + SFA 4 + SFB 8 -> next power of two
  static constexpr int TMEM_NEED = BN + 12;
  static constexpr int TMEM_COLS = TMEM_NEED <= 32 ? 32 : TMEM_NEED <= 64 ? 64 : TMEM_NEED <= 128 ? 128
                                   : TMEM_NEED <= 256 ? 256 : 512;
  static constexpr int SFA_COL = BN;
  static constexpr int SFB_COL = BN + 4;
  static constexpr int SMEM_BYTES = 1024 /*align slack*/ + STAGES * STAGE_BYTES + 1024 /*barriers*/;
  static_assert(STAGES >= 2, "not enough shared memory for two stages");
  static_assert(BN * BM * 4 <= STAGES * STAGE_BYTES, "split-K partial tile must fit in stage smem");
};

__host__ __device__ constexpr uint32_t make_idesc(int bn, int sf_id, int wfmt = 0) {
  return (0u << 4)                       // b_sf_id set below
         | (w_mma_format(wfmt) << 7)     // A format: the weight element type
         | (0u << 10)                    // B format: E4M3
         | ((uint32_t)(bn >> 3) << 17)   // N >> 3
         | (1u << 23)                    // scale format UE8M0
         | ((uint32_t)(BM >> 4) << 24)   // M >> 4
         | ((uint32_t)sf_id << 29)       // A scale-factor id (byte within the TMEM word)
         | ((uint32_t)sf_id << 4);       // B scale-factor id
}

// Producer fused into the decode GEMM (ACT > 0, BN = 16, single row tile): the four epilogue
// warps build the e4m3 activation tiles themselves instead of a separate producer kernel.
//   ACT 1 (norm): s = x (+ res); y = bf16(s * rsqrt(mean(s^2) + eps) * (1 + w)); res_out = bf16(s)
//   ACT 2 (silu): y = bf16(silu(g) * u) with x = [g | u] (K columns each)
// then q = e4m3(y / scale), scale = max(amax(y) / 448, 1 / (448 * 512)) per row -- the exact
// numerics of the stand-alone producers (norm_quant.cu).
constexpr int kActMaxChunks = 9;       // fused producers: rows of up to 9 * 1024 features

struct ActArgs {
  const __nv_bfloat16* x;
  int ldx;
  const __nv_bfloat16* res;
  int ldr;
  const __nv_bfloat16* w;
  __nv_bfloat16* res_out;
  int ldro;
  float eps;
  int K;
};

DEVI void act_load8(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// 8 activation values of row m at feature k (k % 8 == 0): y (bf16-rounded) and, for norm, the
// residual sum s
template <int ACT>
DEVI void act_values(const ActArgs& aa, int m, int k, float rs, float (&y)[8], float (&sv)[8]) {
  if constexpr (ACT == 1) {
    act_load8(aa.x + (size_t)m * aa.ldx + k, sv);
    if (aa.res) {
      float r[8];
      act_load8(aa.res + (size_t)m * aa.ldr + k, r);
#pragma unroll
      for (int j = 0; j < 8; ++j) sv[j] += r[j];
    }
    float wv[8];
    act_load8(aa.w + k, wv);
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = bf16_round(sv[j] * rs * (wv[j] + 1.f));
  } else {
    float g[8], u[8];
    act_load8(aa.x + (size_t)m * aa.ldx + k, g);
    act_load8(aa.x + (size_t)m * aa.ldx + aa.K + k, u);
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = bf16_round(g[j] / (1.f + __expf(-g[j])) * u[j]);
  }
}

// sum over the 128 producer threads (warps 2-5), named barrier 2
DEVI float prod_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = (threadIdx.x >> 5) - 2;
  asm volatile("bar.sync 2, 128;" ::: "memory");
  if ((threadIdx.x & 31) == 0) red[w] = v;
  asm volatile("bar.sync 2, 128;" ::: "memory");
  return red[0] + red[1] + red[2] + red[3];
}
DEVI float prod_max(float v, float* red) {
  v = warp_max(v);
  const int w = (threadIdx.x >> 5) - 2;
  asm volatile("bar.sync 2, 128;" ::: "memory");
  if ((threadIdx.x & 31) == 0) red[w] = v;
  asm volatile("bar.sync 2, 128;" ::: "memory");
  return fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
}

// RS: reduce-scatter push for the prefill two-shot all-reduce (comm_ts.cu): output row m goes to
// its owner's source slot (push.peer[o], o = m / per with per = push.half_words, row length
// push.ld) as bf16 pairs; once the CTA's stores are fenced it adds 1 to every owner's arrival
// counter of this rank.
constexpr int kTsHeader = 8192;   // comm_ts.cu buffer header bytes

DEVI void rs_store(const PushArgs& pa, int m, int n, float lo, float hi) {
  const int per = (int)pa.half_words;
  const int o = m / per;
  __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(pa.peer[o] + kTsHeader) +
                       ((size_t)pa.rank * per + (m - o * per)) * pa.ld + n;
  *reinterpret_cast<__nv_bfloat162*>(dst) = __floats2bfloat162_rn(lo, hi);
}

// FIN (decode, BN = 16): the CTA that arrives last on a self-resetting counter, after every CTA
// has written its output rows, runs the next linear's producer over the whole rows (finish.cuh):
// residual add + RMSNorm(1 + w) + e4m3, or SiLU * mul + e4m3.
struct FinCtl {
  unsigned* done;   // arrival counter (zero, self-resetting)
  FinArgs args;
};

template <int BN, bool GROUPED = false, bool PUSH = false, int ACT = 0, bool RS = false, int FIN = 0>
__global__ void __launch_bounds__(kThreads, Cfg<BN>::MIN_BLOCKS)
    mxfp4_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w,
                      const __grid_constant__ CUtensorMap tmap_a, const uint8_t* __restrict__ sfw,
                      const float* __restrict__ a_scale, __nv_bfloat16* __restrict__ out,
                      int ldo, int M, int N, int K, int wfmt, int k_tiles_per_split, int* __restrict__ status,
                      const int* __restrict__ items, int n_per_group, const PushArgs push,
                      const ActArgs act, const FinCtl fin) {
  using C = Cfg<BN>;
  // Grouped (MoE) mode: blockIdx.y indexes a work table of (expert, first row, rows); the
  // expert's weights are rows [e * n_per_group, (e + 1) * n_per_group) of the stacked tensor.
  int g_expert = 0, g_row0 = 0, g_rows = 0;
  if constexpr (GROUPED) {
    pdl_wait();
    g_expert = items[blockIdx.y * 3 + 0];
    g_row0 = items[blockIdx.y * 3 + 1];
    g_rows = items[blockIdx.y * 3 + 2];
    if (g_rows <= 0) return;            // unused slot of the fixed-size work table
  }
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stage_base = smem;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty_bar = full_bar + C::STAGES;
  uint64_t* acc_bar = empty_bar + C::STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_bar + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int n_tile = GROUPED ? (g_expert * (n_per_group / BM) + blockIdx.x) : blockIdx.x;
  const int m_tile = blockIdx.y;
  const int split = blockIdx.z;
  const int num_splits = gridDim.z;
  const int n0 = n_tile * BM;                       // row of the (stacked) weight tensor
  const int m0 = GROUPED ? g_row0 : m_tile * BN;
  const int m_end = GROUPED ? g_row0 + g_rows : M;  // rows of this tile that are stored
  const int n_out0 = GROUPED ? blockIdx.x * BM : n0;  // output column of weight row n0
  const int n_lim = GROUPED ? n_per_group : N;
  const int k_tiles_total = K / BK;
  const int kt0 = split * k_tiles_per_split;
  const int kt1 = min(k_tiles_total, kt0 + k_tiles_per_split);
  const int nk = kt1 - kt0;

  __shared__ float s_act_scale[ACT ? BN : 1];
  __shared__ float s_red[4];
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], ACT ? 2 : 1);   // + the activation producers' arrival
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(acc_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_w);
    if (!ACT) tma_prefetch_desc(&tmap_a);
  }
  pdl_trigger();   // the next kernel may start its own prologue
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  // TMEM address handoff: fence / barrier / fence
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tmem_acc = tmem_base;
  const uint32_t tmem_sfa = tmem_base + C::SFA_COL;
  const uint32_t tmem_sfb = tmem_base + C::SFB_COL;

  // activation scale factors = 1.0 (UE8M0 127) for every lane / byte
  if (warp >= 2) {
    const int q = warp & 3;
    uint32_t ones[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) ones[i] = 0x7F7F7F7Fu;
    tmem_st_32x32b_x8(tmem_sfb + ((uint32_t)(q * 32) << 16), ones);
    tmem_st_wait();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (elect_one()) {
      const uint64_t w_policy = l2_policy_evict_first();   // weights stream once
      const uint8_t* sf_row = sfw + (size_t)n_tile * (size_t)k_tiles_total * SF_TILE_BYTES;
      // Weights and scale factors do not depend on the preceding kernel: fill the pipeline with
      // them while that kernel drains, then wait for it and add the activation tiles.
      const int pre = nk < C::STAGES ? nk : C::STAGES;
      const uint32_t kTx = w_tile_tx(wfmt) + (ACT ? 0 : C::A_TILE_BYTES) + SF_TILE_BYTES;
      for (int i = 0; i < pre; ++i) {
        uint8_t* st = stage_base + i * C::STAGE_BYTES;
        const int kt = kt0 + i;
        mbar_arrive_expect_tx(&full_bar[i], kTx);
        tma_load_2d_hint(st, &tmap_w, &full_bar[i], kt * BK, n0, w_policy);
        bulk_load(st + W_TILE_BYTES + C::A_TILE_BYTES, sf_row + (size_t)kt * SF_TILE_BYTES,
                  SF_TILE_BYTES, &full_bar[i]);
      }
      if (!ACT) {
        pdl_wait();
        for (int i = 0; i < pre; ++i)
          tma_load_2d(stage_base + i * C::STAGE_BYTES + W_TILE_BYTES, &tmap_a, &full_bar[i],
                      (kt0 + i) * BK, m0);
      }
      for (int i = pre; i < nk; ++i) {
        const int s = i % C::STAGES;
        const uint32_t ph = (i / C::STAGES) & 1;
        if (!mbar_wait(&empty_bar[s], ph ^ 1, status)) { *abort_flag = 1; break; }
        uint8_t* st = stage_base + s * C::STAGE_BYTES;
        const int kt = kt0 + i;
        mbar_arrive_expect_tx(&full_bar[s], kTx);
        tma_load_2d_hint(st, &tmap_w, &full_bar[s], kt * BK, n0, w_policy);
        if (!ACT) tma_load_2d(st + W_TILE_BYTES, &tmap_a, &full_bar[s], kt * BK, m0);
        bulk_load(st + W_TILE_BYTES + C::A_TILE_BYTES, sf_row + (size_t)kt * SF_TILE_BYTES,
                  SF_TILE_BYTES, &full_bar[s]);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (elect_one()) {
      pdl_wait();                      // the activation tiles land after the preceding kernel
      bool ok = true;
      for (int i = 0; i < nk; ++i) {
        const int s = i % C::STAGES;
        const uint32_t ph = (i / C::STAGES) & 1;
        if (!mbar_wait(&full_bar[s], ph, status)) { ok = false; *abort_flag = 1; break; }
        tc_fence_after();
        uint8_t* st = stage_base + s * C::STAGE_BYTES;
        const uint32_t w_addr = smem_u32(st);
        const uint32_t a_addr = smem_u32(st + W_TILE_BYTES);
        const uint32_t sf_addr = smem_u32(st + W_TILE_BYTES + C::A_TILE_BYTES);
        // weight scale factors: 32 rows x 16 B atom -> TMEM lanes (x4 quarters), 4 columns
        tmem_cp_32x128b_warpx4(tmem_sfa, sdesc_plain(sf_addr, 0, 128));
#pragma unroll
        for (int kb = 0; kb < BK / 32; ++kb) {
          const uint64_t adesc = sdesc_sw128(w_addr + kb * 32);
          const uint64_t bdesc = sdesc_sw128(a_addr + kb * 32);
          const uint32_t idesc = make_idesc(BN, kb, wfmt);
          mma_mxf8f6f4(tmem_acc, adesc, bdesc, idesc, tmem_sfa | ((uint32_t)kb << 30),
                       tmem_sfb | ((uint32_t)kb << 30), (i > 0 || kb > 0) ? 1u : 0u);
        }
        mma_commit(&empty_bar[s]);     // frees the stage once these MMAs have read it
      }
      if (ok) mma_commit(acc_bar);     // accumulator complete
      else mbar_arrive(acc_bar);
    }
  } else {
    // ---------------- activation producers (ACT) + epilogue ----------------
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;     // weight row within the tile
    const int n = n_out0 + row;        // output column
    pdl_wait();                        // activations / a_scale come from the preceding kernel
    if constexpr (ACT != 0) {
      static_assert(BN == 16, "fused producers run with one 16-row tile");
      // One activation row (M = 1, host-checked).  Thread pt owns the 8-element chunks
      // j = pt + 128 * i of the row (K <= kActMaxChunks * 1024).  All of a thread's loads are
      // issued together; the CTA's own K range is quantised into registers up front, so the
      // pipeline loop below only stores precomputed bytes into each stage's slot.
      constexpr int MAXC = kActMaxChunks;
      const int pt = threadIdx.x - 64;                  // 0..127
      const int Ka = act.K;
      const int nch = Ka / 8;
      const int own0 = kt0 * (BK / 8), own1 = min(kt1 * (BK / 8), nch);
      float rs = 0.f;
      if constexpr (ACT == 1) {
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < MAXC; ++i) {
          const int j = pt + 128 * i;
          if (j < nch) {
            float sv[8];
            act_load8(act.x + j * 8, sv);
            if (act.res) {
              float rr[8];
              act_load8(act.res + j * 8, rr);
#pragma unroll
              for (int e = 0; e < 8; ++e) sv[e] += rr[e];
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) ss += sv[e] * sv[e];
            if (n_tile == 0 && act.res_out && j >= own0 && j < own1) {   // new residual, once
              uint4 o;
              __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
              for (int e = 0; e < 4; ++e) oh[e] = __floats2bfloat162_rn(sv[2 * e], sv[2 * e + 1]);
              *reinterpret_cast<uint4*>(act.res_out + j * 8) = o;
            }
          }
        }
        rs = rsqrtf(prod_sum(ss, s_red) / (float)Ka + act.eps);
      }
      uint32_t ypk[MAXC][4];                            // bf16-rounded y, packed in pairs
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int j = pt + 128 * i;
        if (j < nch) {
          float y[8], sv[8];
          act_values<ACT>(act, 0, j * 8, rs, y, sv);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            __nv_bfloat162 hh = __floats2bfloat162_rn(y[2 * e], y[2 * e + 1]);
            ypk[i][e] = *reinterpret_cast<uint32_t*>(&hh);
            amax = fmaxf(amax, fmaxf(fabsf(y[2 * e]), fabsf(y[2 * e + 1])));
          }
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) ypk[i][e] = 0u;
        }
      }
      amax = prod_max(amax, s_red);
      const float scale = fmaxf(amax / 448.f, 1.f / (448.f * 512.f));
      const float inv = 1.f / scale;
      if (pt == 0) s_act_scale[0] = scale;
      uint2 qv[MAXC];
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        uint16_t* hh = reinterpret_cast<uint16_t*>(&qv[i]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ypk[i][e]));
          hh[e] = f32x2_to_e4m3x2(f.x * inv, f.y * inv);
        }
      }
      // pipeline: stage i holds chunks [kt * 16, kt * 16 + 16) of row 0 (rows 1..15 of the tile
      // are never read back: their output rows are not stored)
      for (int i = 0; i < nk; ++i) {
        const int s = i % C::STAGES;
        const uint32_t ph = (i / C::STAGES) & 1;
        const bool got = mbar_wait(&empty_bar[s], ph ^ 1, status);
        const int jb = (kt0 + i) * (BK / 8);
        const int c = (pt - jb) & 127;                  // chunk of this stage owned by pt, if < 16
        if (got && c < BK / 8) {
          const int j = jb + c;
          uint2 val = make_uint2(0, 0);
#pragma unroll
          for (int ii = 0; ii < MAXC; ++ii)
            if (pt + 128 * ii == j) val = qv[ii];
          uint8_t* slot = stage_base + s * C::STAGE_BYTES + W_TILE_BYTES;
          *reinterpret_cast<uint2*>(slot + (c >> 1) * 16 + (c & 1) * 8) = val;   // row 0: no swizzle
        }
        fence_proxy_async();                            // generic-proxy writes -> tensor core
        if (bar_sync_or(2, 128, !got)) { *abort_flag = 1; break; }   // all four warps leave together
        if (pt == 0) mbar_arrive(&full_bar[s]);
      }
    }
    if (!mbar_wait(acc_bar, 0, status)) *abort_flag = 1;
    tc_fence_after();
    const bool have_acc = nk > 0 && !*abort_flag;
    if (num_splits == 1) {
      const uint32_t seq = PUSH ? push_seq(push) : 0u;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(tmem_acc + ((uint32_t)(q * 32) << 16) + c0, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = m0 + c0 + j;
          if (m >= m_end) break;                       // uniform across the warp
          const float asc = ACT ? s_act_scale[m - m0] : a_scale[m];
          const float v = (have_acc && n < n_lim) ? __uint_as_float(r[j]) * asc : 0.f;
          if constexpr (PUSH) {
            // adjacent lanes own adjacent columns: even lanes store the pair as one LL word
            // straight into this rank's slot of every peer's receive buffer
            const float vn = __shfl_down_sync(0xffffffffu, v, 1);
            if ((lane & 1) == 0 && n < n_lim)
              for (int p = 0; p < push.world; ++p)
                st_ll_pair(push_slot(push, p, seq & 1u, push.rank, M) + (size_t)m * (push.ld / 2) + n / 2,
                           v, vn, seq);
          } else if constexpr (RS) {
            const float vn = __shfl_down_sync(0xffffffffu, v, 1);
            if ((lane & 1) == 0 && n < n_lim) rs_store(push, m, n, v, vn);
          } else if (n < n_lim) {
            out[(size_t)m * ldo + n] = __float2bfloat16_rn(v);
          }
        }
      }
    } else {
      // partial tile -> own shared memory, layout [BN][128] fp32 (stage buffers are idle now)
      float* part = reinterpret_cast<float*>(stage_base);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(tmem_acc + ((uint32_t)(q * 32) << 16) + c0, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) part[(c0 + j) * BM + row] = have_acc ? __uint_as_float(r[j]) : 0.f;
      }
    }
  }

  if (num_splits > 1) {
    // every thread of every CTA in the cluster takes part in both cluster barriers
    __syncwarp();
    cluster_sync();
    if (warp >= 2) {
      const int q = warp & 3;
      const int row = q * 32 + lane;
      const int n = n_out0 + row;
      const uint32_t my_rank = cluster_ctarank();
      const uint32_t part_addr = smem_u32(stage_base);
      const uint32_t seq = PUSH ? push_seq(push) : 0u;
      for (int j = my_rank; j < BN; j += num_splits) {
        const int m = m0 + j;
        if (m >= m_end) break;                         // uniform across the warp
        float acc = 0.f;
        if (n < n_lim) {
          for (int r = 0; r < num_splits; ++r) {
            const uint32_t a = mapa_shared(part_addr + (uint32_t)((j * BM + row) * 4), (uint32_t)r);
            float v;
            asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a));
            acc += v;
          }
          acc *= ACT ? s_act_scale[m - m0] : a_scale[m];
        }
        if constexpr (PUSH) {
          const float vn = __shfl_down_sync(0xffffffffu, acc, 1);
          if ((lane & 1) == 0 && n < n_lim)
            for (int p = 0; p < push.world; ++p)
              st_ll_pair(push_slot(push, p, seq & 1u, push.rank, M) + (size_t)m * (push.ld / 2) + n / 2,
                         acc, vn, seq);
        } else if constexpr (RS) {
          const float vn = __shfl_down_sync(0xffffffffu, acc, 1);
          if ((lane & 1) == 0 && n < n_lim) rs_store(push, m, n, acc, vn);
        } else if (n < n_lim) {
          out[(size_t)m * ldo + n] = __float2bfloat16_rn(acc);
        }
      }
    }
    __syncwarp();
    cluster_sync();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  if constexpr (FIN != 0) {
    __shared__ bool s_fin;
    __shared__ float s_fred[kThreads / 32];
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned total = gridDim.x * gridDim.y * gridDim.z;
      s_fin = atomicAdd(fin.done, 1u) == total - 1u;
      if (s_fin) *fin.done = 0u;
    }
    __syncthreads();
    if (s_fin) {     // every CTA's rows are written: finish them with all six warps
      __threadfence();
      float* buf = reinterpret_cast<float*>(stage_base);
      for (int m = 0; m < M; ++m) finish_row<kThreads, FIN>(fin.args, out, ldo, N, m, buf, s_fred);
    }
  }
  if constexpr (RS) {
    // this CTA's rows are stored in their owners' slots: one arrival at every owner
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0)
      for (int o = 0; o < push.world; ++o)
        asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(
                         reinterpret_cast<uint32_t*>(push.peer[o]) + push.rank),
                     "r"(1u) : "memory");
  }
}

// ---------------------------------------------------------------------------------------------
// Prefill tiles on CTA pairs (tcgen05 cta_group::2).  A 2-CTA cluster owns a 256 x 256 output
// tile: each CTA stages its 128 weight rows and its 128 of the 256 tokens, and the pair's leader
// issues one M = 256, N = 256 block-scaled MMA per 32 K.  Against one CTA per 128 x 256 tile this
// halves the activation bytes each SM moves through shared memory per MMA -- the limit of the
// fp8-rate MMA with both operands in shared memory.  The kernel is persistent (one pair per two
// SMs, tiles strided by the pair count, weight tiles fastest so concurrent pairs share the
// activation tile in L2); the producers keep prefetching the next tile's stages while the
// epilogue drains the accumulator.  No load is multicast: each CTA's TMA fills its own shared
// memory and signals the leader's barrier (.cta_group::2 form).
// ---------------------------------------------------------------------------------------------
constexpr int P_WROWS = 2 * BM;                            // weight rows per pair tile (MMA M)
constexpr int P_BN = 224;                                  // tokens per pair tile (MMA N)
constexpr int P_HALF = P_BN / 2;                           // tokens staged per CTA
constexpr int P_W_BYTES = BM * BK;                         // expanded weight tile (16 KB)
constexpr int P_A_BYTES = P_HALF * BK;                     // this CTA's activation half
constexpr int P_STAGE = (P_W_BYTES + P_A_BYTES + SF_TILE_BYTES + 1023) / 1024 * 1024;
constexpr int P_STAGES = (kSmemBudget - 2048) / P_STAGE;
constexpr int P_SMEM = 1024 + P_STAGES * P_STAGE + 1024;
// TMEM: two accumulators (the epilogue drains one while the MMAs fill the other), then the
// weight scale factors and 32 columns of UE8M0 1.0 for the activations
constexpr int P_TMEM_COLS = 512;
constexpr int P_SFA_COL = 2 * P_BN;
constexpr int P_SFB_COL = P_SFA_COL + 8;
static_assert(P_SFB_COL + 32 <= P_TMEM_COLS, "TMEM columns");
static_assert(P_HALF % 8 == 0, "activation half tile in whole 8-row swizzle atoms");
static_assert(P_STAGES >= 4, "pair pipeline depth");

struct PairBars {
  uint64_t full[P_STAGES];      // leader: both CTAs' bytes of a stage landed
  uint64_t empty[P_STAGES];     // each CTA: the pair's MMAs have read its stage
  uint64_t acc_full[2];         // each CTA: accumulator b of the tile is complete
  uint64_t acc_empty[2];        // leader: both epilogues drained accumulator b
  uint32_t tmem;
  int abort;
};

__host__ __device__ constexpr uint32_t make_idesc_pair(int sf_id, int wfmt) {
  return (w_mma_format(wfmt) << 7)             // A format: the weight element type
         | (0u << 10)                          // B format: E4M3
         | ((uint32_t)(P_BN >> 3) << 17)       // N >> 3
         | (1u << 23)                          // scale format UE8M0
         | ((uint32_t)(P_WROWS >> 4) << 24)    // M >> 4 (the pair's 256 rows)
         | ((uint32_t)sf_id << 29) | ((uint32_t)sf_id << 4);
}

DEVI void tma_load_2d_pair(void* smem_dst, const void* desc, uint32_t mbar, int c0, int c1,
                           uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(desc), "r"(mbar), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}
DEVI void mma_mxf8f6f4_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                            uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}
// arrive on the mbarrier at a cluster address once the pair's prior tcgen05 ops are done
DEVI void commit_pair(uint32_t mbar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   mbar)
               : "memory");
}
DEVI void tmem_cp_pair_32x128b_warpx4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc)
               : "memory");
}
DEVI void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
DEVI void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
DEVI void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
DEVI void mbar_arrive_cluster(uint32_t mbar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(mbar) : "memory");
}

// Warp roles as in the one-CTA kernel: warp 0 = TMA producer (both CTAs), warp 1 = TMEM
// allocator (both CTAs) and MMA issuer (leader only), warps 2..5 = epilogue (both CTAs, each its
// own 128 weight rows x 256 tokens of the accumulator).
template <bool RS>
__global__ void __launch_bounds__(kThreads, 1) gemm_pair_kernel(
    const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
    const __grid_constant__ CUtensorMap tmap_sf, const float* __restrict__ a_scale,
    __nv_bfloat16* __restrict__ out, int ldo, int M, int N, int Kw, int wfmt,
    int* __restrict__ status, const PushArgs push) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PairBars* bars = reinterpret_cast<PairBars*>(smem + P_STAGES * P_STAGE);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();             // 0 = leader (issues the MMAs)
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int n_tiles = (N + P_WROWS - 1) / P_WROWS;
  const int num_tiles = n_tiles * ((M + P_BN - 1) / P_BN);
  const int k_tiles = Kw / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->acc_full[b], 1);
      mbar_init(&bars->acc_empty[b], 2);
    }
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_sf);
  }
  pdl_trigger();
  if (warp == 1) {
    tmem_alloc_pair(&bars->tmem, P_TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_acc = bars->tmem;
  const uint32_t tmem_sfa = tmem_acc + P_SFA_COL;
  const uint32_t tmem_sfb = tmem_acc + P_SFB_COL;
  // a failed wait stops both CTAs of the pair: the flag is raised here and in the partner
  const uint32_t abort_peer = mapa_shared(smem_u32(&bars->abort), rank ^ 1u);
  auto pair_abort = [&]() {
    *(volatile int*)&bars->abort = 1;
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(abort_peer), "r"(1) : "memory");
  };
  if (warp >= 2) {              // activation scale factors: UE8M0 1.0 everywhere
    const int q = warp & 3;
    uint32_t ones[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) ones[i] = 0x7F7F7F7Fu;
#pragma unroll
    for (int c = 0; c < 32; c += 8) tmem_st_32x32b_x8(tmem_sfb + ((uint32_t)(q * 32) << 16) + c, ones);
    tmem_st_wait();
  }
  tc_fence_before();
  __syncthreads();
  __syncwarp();
  cluster_sync();               // both CTAs: barriers initialised, TMEM allocated and filled
  tc_fence_after();

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (elect_one()) {
      const uint64_t w_policy = l2_policy_evict_first();
      const uint64_t a_policy = l2_policy_evict_last();
      const uint32_t tx = 2u * (w_tile_tx(wfmt) + P_A_BYTES + SF_TILE_BYTES);
      pdl_wait();
      uint32_t it = 0;
      for (int t = pair; t < num_tiles && !*(volatile int*)&bars->abort; t += npairs) {
        const int n0 = (t % n_tiles) * P_WROWS + (int)rank * BM;
        const int m0 = (t / n_tiles) * P_BN + (int)rank * P_HALF;
        for (int kt = 0; kt < k_tiles; ++kt, ++it) {
          const int s = it % P_STAGES;
          const uint32_t ph = (it / P_STAGES) & 1;
          if (!mbar_wait(&bars->empty[s], ph ^ 1, status)) { pair_abort(); break; }
          uint8_t* st = smem + s * P_STAGE;
          const uint32_t full = mapa_shared(smem_u32(&bars->full[s]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&bars->full[s], tx);
          tma_load_2d_pair(st, &tmap_w, full, kt * BK, n0, w_policy);
          tma_load_2d_pair(st + P_W_BYTES, &tmap_a, full, kt * BK, m0, a_policy);
          tma_load_2d_pair(st + P_W_BYTES + P_A_BYTES, &tmap_sf, full, 0, (n0 / BM) * k_tiles + kt,
                           w_policy);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader) ----------------
    if (rank == 0 && elect_one()) {
      pdl_wait();                                     // the producers' tiles follow it
      const uint32_t empty_peer0 = mapa_shared(smem_u32(&bars->empty[0]), 1);
      const uint32_t accf_peer0 = mapa_shared(smem_u32(&bars->acc_full[0]), 1);
      uint32_t it = 0, tc = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok && !*(volatile int*)&bars->abort; t += npairs, ++tc) {
        const int ab = tc & 1;                        // accumulator of this tile
        if (!mbar_wait(&bars->acc_empty[ab], ((tc >> 1) & 1) ^ 1, status)) { ok = false; break; }
        tc_fence_after();
        for (int kt = 0; kt < k_tiles; ++kt, ++it) {
          const int s = it % P_STAGES;
          const uint32_t ph = (it / P_STAGES) & 1;
          if (!mbar_wait(&bars->full[s], ph, status)) { ok = false; break; }
          tc_fence_after();
          uint8_t* st = smem + s * P_STAGE;
          const uint32_t w_addr = smem_u32(st);
          const uint32_t a_addr = smem_u32(st + P_W_BYTES);
          tmem_cp_pair_32x128b_warpx4(tmem_sfa, sdesc_plain(smem_u32(st + P_W_BYTES + P_A_BYTES), 0, 128));
#pragma unroll
          for (int kb = 0; kb < BK / 32; ++kb)
            mma_mxf8f6f4_pair(tmem_acc + (uint32_t)(ab * P_BN), sdesc_sw128(w_addr + kb * 32),
                              sdesc_sw128(a_addr + kb * 32),
                              make_idesc_pair(kb, wfmt), tmem_sfa | ((uint32_t)kb << 30),
                              tmem_sfb | ((uint32_t)kb << 30), (kt > 0 || kb > 0) ? 1u : 0u);
          commit_pair(smem_u32(&bars->empty[s]));
          commit_pair(empty_peer0 + (uint32_t)(s * sizeof(uint64_t)));
        }
        if (!ok) break;
        commit_pair(smem_u32(&bars->acc_full[ab]));
        commit_pair(accf_peer0 + (uint32_t)(ab * sizeof(uint64_t)));
      }
      if (!ok) pair_abort();
    }
  } else {
    // ---------------- epilogue (both CTAs) ----------------
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t acc_empty0 = mapa_shared(smem_u32(&bars->acc_empty[0]), 0);
    const uint32_t lane_base0 = tmem_acc + ((uint32_t)(q * 32) << 16);
    pdl_wait();
    uint32_t tc = 0;
    for (int t = pair; t < num_tiles; t += npairs, ++tc) {
      const int ab = tc & 1;
      const uint32_t lane_base = lane_base0 + (uint32_t)(ab * P_BN);
      const bool got = mbar_wait(&bars->acc_full[ab], (tc >> 1) & 1, status);
      if (!got) pair_abort();
      tc_fence_after();
      const int n = (t % n_tiles) * P_WROWS + (int)rank * BM + row;
      const int mt0 = (t / n_tiles) * P_BN;
      auto store16 = [&](const uint32_t (&r)[16], int c) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = mt0 + c * 16 + j;
          if (m >= M) break;                               // uniform across the warp
          const float v = got ? __uint_as_float(r[j]) * a_scale[m] : 0.f;
          if constexpr (RS) {
            const float vn = __shfl_down_sync(0xffffffffu, v, 1);
            if ((lane & 1) == 0 && n < N) rs_store(push, m, n, v, vn);
          } else if (n < N) {
            out[(size_t)m * ldo + n] = __float2bfloat16_rn(v);
          }
        }
      };
      uint32_t ra[16], rb[16];
      tmem_ld_32x32b_x16(lane_base, ra);
      tmem_ld_wait();
#pragma unroll 1
      for (int c = 0; c < P_BN / 16; c += 2) {
        tmem_ld_32x32b_x16(lane_base + (uint32_t)((c + 1) * 16), rb);
        store16(ra, c);
        tmem_ld_wait();
        if (c + 2 < P_BN / 16) tmem_ld_32x32b_x16(lane_base + (uint32_t)((c + 2) * 16), ra);
        store16(rb, c + 1);
        tmem_ld_wait();
      }
      // the accumulator is free for the pair's next tile once all four warps have read it
      tc_fence_before();
      const bool stop = bar_sync_or(1, 128, *(volatile int*)&bars->abort != 0);
      if (threadIdx.x == 64) mbar_arrive_cluster(acc_empty0 + (uint32_t)(ab * sizeof(uint64_t)));
      if (stop) break;                                 // the same answer in all four warps
    }
  }

  tc_fence_before();
  __syncthreads();
  __syncwarp();
  cluster_sync();               // the pair's MMAs, copies and remote arrivals are all done
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_acc, P_TMEM_COLS);
  }
  if constexpr (RS) {
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0)
      for (int o = 0; o < push.world; ++o)
        asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(
                         reinterpret_cast<uint32_t*>(push.peer[o]) + push.rank),
                     "r"(1u) : "memory");
  }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
struct MapKey {
  uintptr_t ptr;
  int64_t rows, cols, stride;
  int box_rows;
  int wfmt;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && rows == o.rows && cols == o.cols && stride == o.stride &&
           box_rows == o.box_rows && wfmt == o.wfmt;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<uintptr_t>()(k.ptr) ^ (std::hash<int64_t>()(k.rows) << 1) ^
           (std::hash<int64_t>()(k.cols) << 7) ^ (std::hash<int>()(k.box_rows) << 13);
  }
};

static std::mutex g_map_mu;
static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_wmaps;

// Weight element type and whole-tile K from the stored row width (bytes) and the activation's K:
// the three packings give distinct widths for the same K tiles, so the width names the type.
struct WFmt {
  int code;
  int Kw;
};
static WFmt weight_fmt(int64_t row_bytes, int K) {
  const int64_t Kp = (int64_t)(K + BK - 1) / BK * BK;
  if (row_bytes * 2 == Kp) return {0, (int)Kp};
  if (row_bytes * 4 == Kp * 3) return {1, (int)Kp};
  if (row_bytes == Kp) return {2, (int)Kp};
  TORCH_CHECK(false, "MX weight: a row of ", row_bytes, " bytes is not K = ", Kp,
              " (activation K rounded up to 128) as e2m1, e2m3 or e4m3");
  return {0, 0};
}

static CUtensorMap weight_map(const torch::Tensor& packed, int64_t N, int64_t K, int wfmt = 0) {
  MapKey key{(uintptr_t)packed.data_ptr(), N, K, packed.stride(0), BM, wfmt};
  std::lock_guard<std::mutex> g(g_map_mu);
  auto it = g_wmaps.find(key);
  if (it != g_wmaps.end()) return it->second;
  const CUtensorMapDataType dt = wfmt == 0 ? CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B
                                 : wfmt == 1 ? CU_TENSOR_MAP_DATA_TYPE_16U6_ALIGN16B
                                             : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  CUtensorMap m = make_tma_2d(packed.data_ptr(), dt,
                              /*inner elems*/ K, /*rows*/ N, /*row stride bytes*/ packed.stride(0),
                              /*box inner*/ BK, /*box rows*/ BM, CU_TENSOR_MAP_SWIZZLE_128B);
  g_wmaps.emplace(key, m);
  return m;
}

template <int BN>
static void launch(const torch::Tensor& a, const torch::Tensor& a_scale, const torch::Tensor& wp,
                   const torch::Tensor& sf, torch::Tensor& out, int M, int N, int K, int splits,
                   int* status, cudaStream_t stream, const PushArgs& push, int act_mode = 0,
                   const ActArgs& aa = ActArgs{}, bool rs = false, int fin_mode = 0,
                   const FinCtl& fc = FinCtl{}) {
  using C = Cfg<BN>;
  const WFmt wf = weight_fmt(wp.size(1), K);   // whole K tiles of stored weight
  const int Kw = wf.Kw;
  CUtensorMap tw = weight_map(wp, N, Kw, wf.code);
  // fused producers build the activation tiles in the kernel: no activation tensor map
  CUtensorMap ta = act_mode ? tw
                            : make_tma_2d(a.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, K, M,
                                          a.stride(0), BK, BN, CU_TENSOR_MAP_SWIZZLE_128B);
  const int k_tiles = Kw / BK;
  const int per = (k_tiles + splits - 1) / splits;
  dim3 grid((N + BM - 1) / BM, (M + BN - 1) / BN, splits);
  using KernT = decltype(&mxfp4_gemm_kernel<BN, false, false, 0>);
  KernT kern = push.world ? mxfp4_gemm_kernel<BN, false, true, 0> : mxfp4_gemm_kernel<BN, false, false, 0>;
  int variant = push.world ? 1 : 0;
  if (rs) { kern = mxfp4_gemm_kernel<BN, false, false, 0, true>; variant = 4; }
  if constexpr (BN == 16) {
    if (act_mode == 1) { kern = mxfp4_gemm_kernel<BN, false, false, 1>; variant = 2; }
    if (act_mode == 2) { kern = mxfp4_gemm_kernel<BN, false, false, 2>; variant = 3; }
    if (fin_mode == kFinNorm) { kern = mxfp4_gemm_kernel<BN, false, false, 0, false, kFinNorm>; variant = 5; }
    if (fin_mode == kFinSilu) { kern = mxfp4_gemm_kernel<BN, false, false, 0, false, kFinSilu>; variant = 6; }
  } else {
    TORCH_CHECK(act_mode == 0 && fin_mode == 0, "fused producers / finishers need a 16-row tile");
  }
  static bool attr_set[7] = {false, false, false, false, false, false, false};
  if (!attr_set[variant]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES));
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    attr_set[variant] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = 1;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = splits;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  const bool no_out = push.world || rs;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, tw, ta, (const uint8_t*)sf.data_ptr(),
                                    act_mode ? (const float*)nullptr : (const float*)a_scale.data_ptr(),
                                    no_out ? nullptr : (__nv_bfloat16*)out.data_ptr(),
                                    no_out ? 0 : (int)out.stride(0), M, N, Kw, wf.code,
                                    per, status, (const int*)nullptr, 0, push, aa, fc));
}

// scale-factor tiles as TMA rows: 512 bytes (128 x u32) per (128-row tile, k tile)
static CUtensorMap sf_map(const torch::Tensor& sf, int64_t rows) {
  MapKey key{(uintptr_t)sf.data_ptr(), rows, 128, 512, 1, -1};
  std::lock_guard<std::mutex> g(g_map_mu);
  auto it = g_wmaps.find(key);
  if (it != g_wmaps.end()) return it->second;
  CUtensorMap m = make_tma_2d(sf.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT32, 128, rows, 512, 128, 1,
                              CU_TENSOR_MAP_SWIZZLE_NONE);
  g_wmaps.emplace(key, m);
  return m;
}

static bool pair_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("RADIANCE_GEMM_PAIR");
    return !(e && e[0] == '0');
  }();
  return on;
}
constexpr int kPairMinRows = 512;      // prefill chunks; shorter batches keep the one-CTA tiles

// Persistent CTA-pair GEMM (prefill).  Returns the CTA count (the RS arrival count).
template <bool RS>
static int launch_pair(const torch::Tensor& a, const torch::Tensor& a_scale, const torch::Tensor& wp,
                       const torch::Tensor& sf, torch::Tensor& out, int M, int N, int K,
                       int* status, cudaStream_t stream, const PushArgs& push) {
  const WFmt wf = weight_fmt(wp.size(1), K);
  const int Kw = wf.Kw;
  const int k_tiles = Kw / BK;
  TORCH_CHECK(sf.numel() >= (int64_t)((N + BM - 1) / BM) * k_tiles * SF_TILE_BYTES,
              "mxfp4_gemm: scale-factor tiles");
  CUtensorMap tw = weight_map(wp, N, Kw, wf.code);
  CUtensorMap ta = make_tma_2d(a.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, K, M, a.stride(0), BK,
                               P_HALF, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap ts = sf_map(sf, (int64_t)((N + BM - 1) / BM) * k_tiles);
  static int sms = [] {
    int dev = 0, v = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
  }();
  const int tiles = ((N + P_WROWS - 1) / P_WROWS) * ((M + P_BN - 1) / P_BN);
  const int pairs = std::max(1, std::min(tiles, sms / 2));
  auto kern = gemm_pair_kernel<RS>;
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM));
    attr = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = P_SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = 2;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, tw, ta, ts, (const float*)a_scale.data_ptr(),
                                    RS ? nullptr : (__nv_bfloat16*)out.data_ptr(),
                                    RS ? 0 : (int)out.stride(0), M, N, Kw, wf.code, status, push));
  return 2 * pairs;
}

static int pick_splits(int tiles, int k_tiles, int ctas_per_sm) {
  // fill the SMs in one wave: grow the cluster along K while the grid fits the resident slots
  // (148 SMs x CTAs per SM) and each CTA keeps >= 4 k-tiles.  Powers of two only: clusters of 7
  // (280 CTAs for out_proj / down) measured slower than 4 (10.1 vs 6.6 us, 11.9 vs 8.0 us at M = 1)
  // -- a 7-CTA cluster leaves SMs of a GPC unusable for the next one.
  const int slots = 148 * ctas_per_sm;
  int s = 1;
  while (s < 8 && tiles * s * 2 <= slots && k_tiles / (s * 2) >= 4) s *= 2;
  return s;
}

template <int BN>
static void launch_grouped(const torch::Tensor& a, const torch::Tensor& a_scale,
                           const torch::Tensor& wp, const torch::Tensor& sf, torch::Tensor& out,
                           const torch::Tensor& items, int max_items, int n_per_group, int K,
                           int* status, cudaStream_t stream) {
  using C = Cfg<BN>;
  const int M = a.size(0);
  const int Ntot = wp.size(0);
  const WFmt wf = weight_fmt(wp.size(1), K);
  CUtensorMap tw = weight_map(wp, Ntot, K, wf.code);
  CUtensorMap ta = make_tma_2d(a.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, K, M, a.stride(0), BK,
                               BN, CU_TENSOR_MAP_SWIZZLE_128B);
  auto kern = mxfp4_gemm_kernel<BN, true>;
  static bool attr_set = false;
  if (!attr_set) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES));
    attr_set = true;
  }
  dim3 grid(n_per_group / BM, max_items, 1);
  C10_CUDA_CHECK(launch_pdl(kern, grid, dim3(kThreads), C::SMEM_BYTES, stream, tw, ta,
                            (const uint8_t*)sf.data_ptr(), (const float*)a_scale.data_ptr(),
                            (__nv_bfloat16*)out.data_ptr(), (int)out.stride(0), M, Ntot, K,
                            wf.code, K / BK, status, (const int*)items.data_ptr(), n_per_group, PushArgs{},
                            ActArgs{}, FinCtl{}));
}

}  // namespace mxfp4

// Grouped (MoE) MX GEMM.  a: expert-sorted e4m3 rows [R, K]; wp/sf: stacked expert weights
// [E*n_per_group, K * bits / 8]; items [max_items, 3] int32 = (expert, first row, rows), rows <= bn.
void mxfp4_grouped_gemm(torch::Tensor a, torch::Tensor a_scale, torch::Tensor wp, torch::Tensor sf,
                        torch::Tensor out, torch::Tensor items, int64_t bn, int64_t n_per_group,
                        torch::Tensor status) {
  using namespace mxfp4;
  TORCH_CHECK(a.scalar_type() == at::kFloat8_e4m3fn && out.scalar_type() == at::kBFloat16, "dtypes");
  const int K = a.size(1);
  TORCH_CHECK(K % BK == 0 && n_per_group % BM == 0, "grouped gemm: K % 128 and N % 128");
  const int max_items = items.size(0);
  if (a.size(0) == 0 || max_items == 0) return;
  const at::cuda::CUDAGuard guard(a.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  int* st = status.numel() ? status.data_ptr<int>() : nullptr;
  switch (bn) {
    case 16: launch_grouped<16>(a, a_scale, wp, sf, out, items, max_items, n_per_group, K, st, stream); break;
    case 32: launch_grouped<32>(a, a_scale, wp, sf, out, items, max_items, n_per_group, K, st, stream); break;
    case 64: launch_grouped<64>(a, a_scale, wp, sf, out, items, max_items, n_per_group, K, st, stream); break;
    case 128: launch_grouped<128>(a, a_scale, wp, sf, out, items, max_items, n_per_group, K, st, stream); break;
    default: launch_grouped<256>(a, a_scale, wp, sf, out, items, max_items, n_per_group, K, st, stream); break;
  }
}

// a: fp8 e4m3 [M, K] (row stride multiple of 16 bytes), a_scale fp32 [M], wp uint8 [N, Kw * bits
// / 8] (e2m1 4, e2m3 6, e4m3 8 bits an element; Kw = K rounded up to 128),
// sf: tiled scale factors, out: bf16 [M, N] (row stride ldo) -- or, with push.world > 0, no
// output tensor: the tiles go to the peers' receive buffers.  Returns the number of output
// tiles (= arrivals each peer receives from this rank).
static int64_t mxfp4_gemm_impl(torch::Tensor a, torch::Tensor a_scale, torch::Tensor wp,
                               torch::Tensor sf, torch::Tensor out, int64_t splits_override,
                               torch::Tensor status, const PushArgs& push, bool rs = false) {
  using namespace mxfp4;
  const bool has_out = !push.world && !rs;
  TORCH_CHECK(a.is_cuda() && wp.is_cuda() && (!has_out || out.is_cuda()),
              "mxfp4_gemm: CUDA tensors required");
  TORCH_CHECK(a.scalar_type() == at::kFloat8_e4m3fn, "activations must be float8_e4m3fn");
  TORCH_CHECK(!has_out || out.scalar_type() == at::kBFloat16, "output must be bf16");
  TORCH_CHECK(a.dim() == 2 && a.stride(1) == 1 && (!has_out || out.stride(1) == 1) &&
                  wp.stride(1) == 1, "row-major");
  // K: the activation's input features (a multiple of 32); the stored weight is zero-padded to
  // whole K tiles (Kw), and the activation's missing tail of the last tile is zero-filled by TMA
  // (out-of-range box elements read as zero)
  const int M = a.size(0), K = a.size(1), N = wp.size(0);
  const int Kw = weight_fmt(wp.size(1), K).Kw;
  TORCH_CHECK(K % 32 == 0, "activation K must be a multiple of 32");
  TORCH_CHECK((a.stride(0) % 16) == 0 && (reinterpret_cast<uintptr_t>(a.data_ptr()) % 16) == 0,
              "activation rows must be 16-byte aligned");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(wp.data_ptr()) % 32) == 0 && (wp.stride(0) % 32) == 0,
              "weight rows must be 32-byte aligned");
  if (has_out) TORCH_CHECK(out.size(0) >= M && out.size(1) >= N, "output too small");
  if (M == 0) return 0;
  const at::cuda::CUDAGuard guard(a.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  int* st = status.numel() ? status.data_ptr<int>() : nullptr;
  int bn;
  if (M <= 16) bn = 16;
  else if (M <= 32) bn = 32;
  else if (M <= 64) bn = 64;
  else if (M <= 128) bn = 128;
  else bn = 256;
  const int tiles = ((N + BM - 1) / BM) * ((M + bn - 1) / bn);
  int splits = splits_override > 0 ? (int)splits_override
                                   : pick_splits(tiles, Kw / BK, bn <= 64 ? 2 : 1);
  if (bn == 256 && M >= kPairMinRows && splits_override <= 0 && pair_enabled()) {
    // prefill: persistent CTA-pair tiles (every CTA adds one arrival at every owner for RS)
    if (rs) return launch_pair<true>(a, a_scale, wp, sf, out, M, N, K, st, stream, push);
    launch_pair<false>(a, a_scale, wp, sf, out, M, N, K, st, stream, push);
    return (int64_t)tiles;
  }
  if (rs) {
    // every CTA adds one arrival at every owner: the count the owner waits for
    switch (bn) {
      case 64: launch<64>(a, a_scale, wp, sf, out, M, N, K, splits, st, stream, push, 0, ActArgs{}, true); break;
      case 128: launch<128>(a, a_scale, wp, sf, out, M, N, K, splits, st, stream, push, 0, ActArgs{}, true); break;
      case 256: launch<256>(a, a_scale, wp, sf, out, M, N, K, splits, st, stream, push, 0, ActArgs{}, true); break;
      default: TORCH_CHECK(false, "mxfp4_gemm_rs: more than 32 rows");
    }
    return (int64_t)tiles * splits;
  }
  switch (bn) {
    case 16: launch<16>(a, a_scale, wp, sf, out, M, N, K, splits, st, stream, push); break;
    case 32: launch<32>(a, a_scale, wp, sf, out, M, N, K, splits, st, stream, push); break;
    case 64: launch<64>(a, a_scale, wp, sf, out, M, N, K, splits, st, stream, push); break;
    case 128: launch<128>(a, a_scale, wp, sf, out, M, N, K, splits, st, stream, push); break;
    default: launch<256>(a, a_scale, wp, sf, out, M, N, K, splits, st, stream, push); break;
  }
  return (int64_t)tiles;
}

void mxfp4_gemm(torch::Tensor a, torch::Tensor a_scale, torch::Tensor wp, torch::Tensor sf,
                torch::Tensor out, int64_t splits_override, torch::Tensor status) {
  mxfp4_gemm_impl(a, a_scale, wp, sf, out, splits_override, status, PushArgs{});
}

// Decode GEMM (M <= 16) followed, in the same launch, by the next linear's producer over its
// output rows: fin_mode 1 = residual add + RMSNorm(1 + w) + e4m3 (res optional, res_out optional,
// q [M, N]), 2 = SiLU(g) * u + e4m3 with out = [g | u] (q [M, N / 2]).  ws: int32 [>= 1] zero
// arrival counter (self-resetting).
void mxfp4_gemm_fin(torch::Tensor a, torch::Tensor a_scale, torch::Tensor wp, torch::Tensor sf,
                    torch::Tensor out, int64_t fin_mode, torch::Tensor res, torch::Tensor w,
                    torch::Tensor res_out, torch::Tensor q, torch::Tensor scale, double eps,
                    torch::Tensor ws, torch::Tensor status) {
  using namespace mxfp4;
  TORCH_CHECK(fin_mode == kFinNorm || fin_mode == kFinSilu, "mxfp4_gemm_fin: mode 1 or 2");
  TORCH_CHECK(a.scalar_type() == at::kFloat8_e4m3fn && a.dim() == 2 && a.stride(1) == 1 &&
                  (a.stride(0) % 16) == 0 && (reinterpret_cast<uintptr_t>(a.data_ptr()) % 16) == 0,
              "mxfp4_gemm_fin: e4m3 activation rows, 16-byte aligned");
  const int M = a.size(0), K = a.size(1), N = wp.size(0);
  const int Kw = weight_fmt(wp.size(1), K).Kw;
  TORCH_CHECK(M >= 1 && M <= 16, "mxfp4_gemm_fin: 1..16 rows");
  TORCH_CHECK(K % 32 == 0, "mxfp4_gemm_fin: K");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(wp.data_ptr()) % 32) == 0 && (wp.stride(0) % 32) == 0,
              "mxfp4_gemm_fin: weight rows 32-byte aligned");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(1) == 1 && out.size(0) >= M &&
                  out.size(1) >= N && out.stride(0) % 8 == 0 &&
                  (reinterpret_cast<uintptr_t>(out.data_ptr()) % 16) == 0, "mxfp4_gemm_fin: out");
  const int H = fin_mode == kFinNorm ? N : N / 2;
  TORCH_CHECK(N % 16 == 0 && H * 4 <= Cfg<16>::STAGES * Cfg<16>::STAGE_BYTES, "finisher row length");
  TORCH_CHECK(q.scalar_type() == at::kFloat8_e4m3fn && q.stride(1) == 1 && q.size(0) >= M &&
                  q.size(1) >= H && q.stride(0) % 8 == 0, "mxfp4_gemm_fin: q");
  TORCH_CHECK(scale.scalar_type() == at::kFloat && scale.numel() >= M, "mxfp4_gemm_fin: scale");
  TORCH_CHECK(ws.scalar_type() == at::kInt && ws.numel() >= 1, "mxfp4_gemm_fin: ws");
  FinCtl fc{};
  fc.done = reinterpret_cast<unsigned*>(ws.data_ptr<int>());
  fc.args.q = (uint8_t*)q.data_ptr();
  fc.args.ldq = (int)q.stride(0);
  fc.args.scale = scale.data_ptr<float>();
  fc.args.eps = (float)eps;
  if (fin_mode == kFinNorm) {
    TORCH_CHECK(w.defined() && w.numel() >= N && w.scalar_type() == at::kBFloat16, "norm weight");
    fc.args.w = (const __nv_bfloat16*)w.data_ptr();
    const bool hr = res.defined() && res.numel(), ho = res_out.defined() && res_out.numel();
    TORCH_CHECK(!hr || (res.stride(1) == 1 && res.stride(0) % 8 == 0), "res rows");
    TORCH_CHECK(!ho || (res_out.stride(1) == 1 && res_out.stride(0) % 8 == 0), "res_out rows");
    fc.args.res = hr ? (const __nv_bfloat16*)res.data_ptr() : nullptr;
    fc.args.ldr = hr ? (int)res.stride(0) : 0;
    fc.args.res_out = ho ? (__nv_bfloat16*)res_out.data_ptr() : nullptr;
    fc.args.ldro = ho ? (int)res_out.stride(0) : 0;
  }
  const at::cuda::CUDAGuard guard(a.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  int* st = status.numel() ? status.data_ptr<int>() : nullptr;
  const int tiles = (N + BM - 1) / BM;
  const int splits = pick_splits(tiles, Kw / BK, 2);
  launch<16>(a, a_scale, wp, sf, out, M, N, K, splits, st, stream, PushArgs{}, 0, ActArgs{}, false,
             (int)fin_mode, fc);
}

// Decode GEMM (M <= 16) with its producer fused in: mode 1 = residual add + RMSNorm(1 + w) +
// e4m3 (x = h, res optional, res_out receives the new residual), mode 2 = SiLU(g) * u + e4m3
// (x = [g | u]).  out: bf16 [M, N].
void mxfp4_gemm_act(int64_t mode, torch::Tensor x, torch::Tensor res, torch::Tensor w,
                    torch::Tensor res_out, double eps, torch::Tensor wp, torch::Tensor sf,
                    torch::Tensor out, torch::Tensor status) {
  using namespace mxfp4;
  TORCH_CHECK(mode == 1 || mode == 2, "mxfp4_gemm_act: mode 1 (norm) or 2 (silu)");
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.stride(1) == 1, "x: bf16 rows");
  const int M = x.size(0);
  const int K = mode == 2 ? (int)x.size(1) / 2 : (int)x.size(1);
  const int N = wp.size(0);
  const int Kw = weight_fmt(wp.size(1), K).Kw;
  TORCH_CHECK(M == 1, "mxfp4_gemm_act: one activation row");
  TORCH_CHECK(K <= kActMaxChunks * 1024, "mxfp4_gemm_act: K <= 9216");
  TORCH_CHECK(K % 16 == 0, "mxfp4_gemm_act: K");
  TORCH_CHECK(x.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(x.data_ptr()) % 16) == 0,
              "mxfp4_gemm_act: x rows 16-byte aligned");
  const bool has_res = res.defined() && res.numel();
  const bool has_ro = res_out.defined() && res_out.numel();
  if (mode == 1) {
    TORCH_CHECK(w.numel() >= K, "mxfp4_gemm_act: norm weight");
    TORCH_CHECK(!has_res || (res.stride(0) % 8 == 0 && res.stride(1) == 1), "res rows");
    TORCH_CHECK(!has_ro || (res_out.stride(0) % 8 == 0 && res_out.stride(1) == 1), "res_out rows");
  }
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(1) == 1 && out.size(1) >= N, "out");
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  int* st = status.numel() ? status.data_ptr<int>() : nullptr;
  ActArgs aa{};
  aa.x = (const __nv_bfloat16*)x.data_ptr();
  aa.ldx = (int)x.stride(0);
  aa.res = has_res ? (const __nv_bfloat16*)res.data_ptr() : nullptr;
  aa.ldr = has_res ? (int)res.stride(0) : 0;
  aa.w = mode == 1 ? (const __nv_bfloat16*)w.data_ptr() : nullptr;
  aa.res_out = has_ro ? (__nv_bfloat16*)res_out.data_ptr() : nullptr;
  aa.ldro = has_ro ? (int)res_out.stride(0) : 0;
  aa.eps = (float)eps;
  aa.K = K;
  const int tiles = (N + BM - 1) / BM;
  const int splits = pick_splits(tiles, Kw / BK, 2);
  launch<16>(x, x, wp, sf, out, M, N, K, splits, st, stream, PushArgs{}, (int)mode, aa);
}

// Row-parallel GEMM fused with the reduce-scatter half of the prefill two-shot all-reduce
// (comm_ts.cu): output row m is stored into its owner's slot of this rank in the owner's buffer
// (peers = every rank's two-shot buffer, per = rows per owner).  Returns the CTA count, which is
// the arrival count each owner waits for.
int64_t mxfp4_gemm_rs(torch::Tensor a, torch::Tensor a_scale, torch::Tensor wp, torch::Tensor sf,
                      std::vector<int64_t> peers, int64_t rank, int64_t per, torch::Tensor status) {
  const int world = peers.size();
  TORCH_CHECK(world >= 1 && world <= 8, "rs: world size 1..8");
  TORCH_CHECK(wp.size(0) % 8 == 0, "rs: output features must be a multiple of 8");
  TORCH_CHECK(per * world >= a.size(0) && per % 8 == 0, "rs: rows per owner");
  PushArgs pa{};
  for (int i = 0; i < world; ++i) pa.peer[i] = (uint8_t*)(uintptr_t)peers[i];
  pa.world = world;
  pa.rank = (int)rank;
  pa.half_words = per;
  pa.ld = (int)wp.size(0);
  return mxfp4_gemm_impl(a, a_scale, wp, sf, torch::Tensor(), 0, status, PushArgs{pa}, true);
}

// Row-parallel GEMM fused with the push half of the all-reduce: peers = every rank's receive
// buffer (own included at `rank`), half_words = words of one parity half; slot row = N outputs.
int64_t mxfp4_gemm_push(torch::Tensor a, torch::Tensor a_scale, torch::Tensor wp, torch::Tensor sf,
                        std::vector<int64_t> peers, int64_t rank, int64_t half_words,
                        torch::Tensor status) {
  const int world = peers.size();
  TORCH_CHECK(world >= 1 && world <= 8, "push: world size 1..8");
  TORCH_CHECK(wp.size(0) % 8 == 0, "push: output features must be a multiple of 8");
  TORCH_CHECK((int64_t)world * a.size(0) * (wp.size(0) / 2) <= half_words,
              "push: message exceeds the receive buffer");
  PushArgs pa{};
  for (int i = 0; i < world; ++i) pa.peer[i] = (uint8_t*)(uintptr_t)peers[i];
  pa.world = world;
  pa.rank = (int)rank;
  pa.half_words = half_words;
  pa.ld = (int)wp.size(0);
  return mxfp4_gemm_impl(a, a_scale, wp, sf, torch::Tensor(), 0, status, pa);
}

}  // namespace rad
