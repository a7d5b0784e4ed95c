// Persistent stream-K MXFP4 W4A8 decode GEMM (M <= 16 activation rows) with a fused row finisher.
//
//   C[m, n] = a_scale[m] * sum_k e4m3(A[m, k]) * e2m1(W[n, k]) * 2^(ws[n, k/32] - 127)
//
// Reference behaviour: the split-K decode GEMM of sly/mxfp4/radiance_mxfp4_fp8.hip (:983, fp32
// partials reduced in-kernel by the last block of each n-block through a self-resetting counter,
// :1251-1343) followed by the fused producers (:1835 add_rms_quant, :1941 silu_mul_quant).
//
// B200 design:
//  * One CTA per SM.  The weight matrix is cut into units of one 128-row x 128-K tile (8 KB of
//    packed e2m1); CTA c streams the contiguous unit range [c*U/G, (c+1)*U/G), so every CTA moves
//    the same bytes whatever the shape (stream-K).  A range may start or end inside a 128-row
//    output tile: those tiles are reduced deterministically -- each contributor stores its fp32
//    partial in its own slot and the last one to arrive (self-resetting per-tile counter) sums
//    the slots in contributor order.
//  * The CTA takes about 97 KB of shared memory, so the next kernel's CTA fits beside it: under
//    programmatic dependent launch that CTA fills its own weight pipeline while this kernel
//    finishes, which hides the per-launch pipeline fill.
//  * The weight tile goes through tcgen05.mma.kind::mxf8f6f4.block_scale with the per-32 UE8M0
//    scales copied to tensor memory (tcgen05.cp), accumulators in TMEM (two 16-column buffers, so
//    the MMAs of one tile overlap the epilogue of the previous one).
//  * Finisher: the CTA that completes the last output tile (self-resetting done counter) runs the
//    next layer's producer over the whole output row(s) -- residual add + RMSNorm + e4m3 or
//    SiLU * mul + e4m3 -- so the producer costs no launch and no kernel boundary.
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 TMEM allocator + MMA issuer, warps 2-5
// epilogue (TMEM lane quarter = warp % 4); after the main loop all six warps run the finisher.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "finish.cuh"
#include "tma_host.h"

namespace rad {
namespace gemv {

constexpr int BM = 128;                       // weight rows per tile (MMA M)
constexpr int BK = 128;                       // K per unit (4 MMAs of K = 32)
constexpr int BN = 16;                        // activation rows (MMA N)
constexpr int W_TILE_BYTES = BM * BK;         // padded e2m1 in smem
constexpr int W_TILE_TX = BM * BK / 2;        // packed bytes moved by TMA
constexpr int A_TILE_BYTES = BN * BK;
constexpr int SF_TILE_BYTES = 512;
constexpr int STAGE_BYTES = (W_TILE_BYTES + A_TILE_BYTES + SF_TILE_BYTES + 1023) / 1024 * 1024;
constexpr int STAGES = 5;
constexpr int kThreads = 192;
constexpr int TMEM_COLS = 64;                 // acc 0: [0,16), acc 1: [16,32), SFA 32, SFB 36
constexpr int SFA_COL = 32;
constexpr int SFB_COL = 36;
constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 1024;
constexpr int kMaxFinH = (STAGES * STAGE_BYTES) / 4;   // finisher row buffer (floats)
constexpr int kTileCounters = 4096;           // workspace: per-tile arrival counters
constexpr int kDoneOff = 4096;                // workspace: tiles-done counter
constexpr int kPartOff = 8192;                // workspace: partial slots (fp32), 2 per CTA
static_assert(STAGES * STAGE_BYTES >= BN * BM * 4, "stage memory");

__host__ __device__ constexpr uint32_t make_idesc(int sf_id) {
  return (5u << 7)                       // A format: E2M1
         | (0u << 10)                    // B format: E4M3
         | ((uint32_t)(BN >> 3) << 17)   // N >> 3
         | (1u << 23)                    // scale format UE8M0
         | ((uint32_t)(BM >> 4) << 24)   // M >> 4
         | ((uint32_t)sf_id << 29)       // A scale-factor id
         | ((uint32_t)sf_id << 4);       // B scale-factor id
}

struct GemvArgs {
  const uint8_t* sfw;      // tiled scale factors, 512 B per (tile, k-tile)
  const float* a_scale;    // [M]
  __nv_bfloat16* out;      // [M, N] (row stride ldo); unused with push
  int ldo;
  int M, N;
  int kt;                  // k-tiles per output tile
  int tiles;               // output tiles (ceil(N / 128))
  long long units;         // tiles * kt
  unsigned* tile_cnt;      // [tiles] arrival counters (zero, self-resetting)
  unsigned* done_cnt;      // [1] tiles-done counter (zero, self-resetting)
  float* part;             // [2 * gridDim.x][BN][BM] fp32 partial slots
  int* status;
};

// CTA owning unit u: the largest c with floor(c * U / G) <= u
DEVI int cta_of(long long u, long long U, int G) { return (int)(((u + 1) * G - 1) / U); }
DEVI long long range_lo(int c, long long U, int G) { return (long long)c * U / G; }

template <bool PUSH>
DEVI void write_value(const GemvArgs& g, const PushArgs& push, uint32_t seq, int m, int n, int lane,
                      float v) {
  if constexpr (PUSH) {
    // adjacent lanes own adjacent columns: even lanes store the pair as one LL word into this
    // rank's slot of every peer's receive buffer
    const float vn = __shfl_down_sync(0xffffffffu, v, 1);
    if ((lane & 1) == 0 && n < g.N)
      for (int p = 0; p < push.world; ++p)
        st_ll_pair(push_slot(push, p, seq & 1u, push.rank, g.M) + (size_t)m * (push.ld / 2) + n / 2,
                   v, vn, seq);
  } else {
    if (n < g.N) g.out[(size_t)m * g.ldo + n] = __float2bfloat16_rn(v);
  }
}

template <bool PUSH, int FIN>
__global__ void __launch_bounds__(kThreads, 1)
    gemv_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                const GemvArgs g, const PushArgs push, const FinArgs fin) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stage_base = smem;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* acc_full = empty_bar + STAGES;     // [2]
  uint64_t* acc_empty = acc_full + 2;          // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  __shared__ int s_last;
  __shared__ int s_fin;
  __shared__ float s_red[kThreads / 32];

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int G = gridDim.x, c = blockIdx.x;
  const long long U = g.units;
  const long long u0 = range_lo(c, U, G), u1 = range_lo(c + 1, U, G);
  const int nu = (int)(u1 - u0);
  const int kt = g.kt;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);     // one arrival per epilogue warp
    }
    s_fin = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_a);
  }
  pdl_trigger();   // the next kernel may place its CTA beside this one and fill its pipeline
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tmem_sfa = tmem_base + SFA_COL;
  const uint32_t tmem_sfb = tmem_base + SFB_COL;
  if (warp >= 2) {   // activation scale factors = 1.0 (UE8M0 127) for every lane / byte
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
      constexpr uint32_t kTx = W_TILE_TX + A_TILE_BYTES + SF_TILE_BYTES;
      // weights and scale factors do not depend on the preceding kernel: fill the pipeline with
      // them while it drains, then wait for it and add the activation tiles
      const int pre = nu < STAGES ? nu : STAGES;
      for (int i = 0; i < pre; ++i) {
        const long long u = u0 + i;
        const int t = (int)(u / kt), k = (int)(u % kt);
        uint8_t* st = stage_base + i * STAGE_BYTES;
        mbar_arrive_expect_tx(&full_bar[i], kTx);
        tma_load_2d_hint(st, &tmap_w, &full_bar[i], k * BK, t * BM, w_policy);
        bulk_load(st + W_TILE_BYTES + A_TILE_BYTES, g.sfw + ((size_t)t * kt + k) * SF_TILE_BYTES,
                  SF_TILE_BYTES, &full_bar[i]);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) {
        const int k = (int)((u0 + i) % kt);
        tma_load_2d(stage_base + i * STAGE_BYTES + W_TILE_BYTES, &tmap_a, &full_bar[i], k * BK, 0);
      }
      for (int i = pre; i < nu; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1;
        if (!mbar_wait(&empty_bar[s], ph ^ 1, g.status)) break;
        const long long u = u0 + i;
        const int t = (int)(u / kt), k = (int)(u % kt);
        uint8_t* st = stage_base + s * STAGE_BYTES;
        mbar_arrive_expect_tx(&full_bar[s], kTx);
        tma_load_2d_hint(st, &tmap_w, &full_bar[s], k * BK, t * BM, w_policy);
        tma_load_2d(st + W_TILE_BYTES, &tmap_a, &full_bar[s], k * BK, 0);
        bulk_load(st + W_TILE_BYTES + A_TILE_BYTES, g.sfw + ((size_t)t * kt + k) * SF_TILE_BYTES,
                  SF_TILE_BYTES, &full_bar[s]);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: one accumulation per segment (a run of units of one tile) ----
    if (elect_one()) {
      pdl_wait();                 // the activation tiles land after the preceding kernel
      bool ok = true;
      int seg = 0;
      for (int i = 0; i < nu && ok; ++seg) {
        const long long u = u0 + i;
        const int k0 = (int)(u % kt);
        const int len = min(kt - k0, nu - i);
        const int b = seg & 1;
        if (seg >= 2 && !mbar_wait(&acc_empty[b], ((seg >> 1) - 1) & 1, g.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t acc = tmem_base + b * BN;
        for (int j = 0; j < len; ++j) {
          const int s = (i + j) % STAGES;
          const uint32_t ph = ((i + j) / STAGES) & 1;
          if (!mbar_wait(&full_bar[s], ph, g.status)) { ok = false; break; }
          tc_fence_after();
          uint8_t* st = stage_base + s * STAGE_BYTES;
          const uint32_t w_addr = smem_u32(st);
          const uint32_t a_addr = smem_u32(st + W_TILE_BYTES);
          const uint32_t sf_addr = smem_u32(st + W_TILE_BYTES + A_TILE_BYTES);
          tmem_cp_32x128b_warpx4(tmem_sfa, sdesc_plain(sf_addr, 0, 128));
#pragma unroll
          for (int kb = 0; kb < BK / 32; ++kb)
            mma_mxf8f6f4(acc, sdesc_sw128(w_addr + kb * 32), sdesc_sw128(a_addr + kb * 32),
                         make_idesc(kb), tmem_sfa | ((uint32_t)kb << 30),
                         tmem_sfb | ((uint32_t)kb << 30), (j > 0 || kb > 0) ? 1u : 0u);
          mma_commit(&empty_bar[s]);
        }
        if (ok) mma_commit(&acc_full[b]);
        i += len;
      }
      if (!ok) {   // release the epilogue: it sees the error status and writes zeros
        for (int b = 0; b < 2; ++b) mbar_arrive(&acc_full[b]);
      }
    }
  } else {
    // ---------------- epilogue ----------------
    const int q = warp & 3;
    const int row = q * 32 + lane;
    pdl_wait();                   // a_scale, counters and slots: after the preceding kernel
    const uint32_t seq = PUSH ? push_seq(push) : 0u;
    int seg = 0;
    for (int i = 0; i < nu; ++seg) {
      const long long u = u0 + i;
      const int t = (int)(u / kt), k0 = (int)(u % kt);
      const int len = min(kt - k0, nu - i);
      const int b = seg & 1;
      const bool got = mbar_wait(&acc_full[b], (seg >> 1) & 1, g.status);
      tc_fence_after();
      uint32_t r[16];
      tmem_ld_32x32b_x16(tmem_base + ((uint32_t)(q * 32) << 16) + b * BN, r);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
      if (!got) {
#pragma unroll
        for (int j = 0; j < 16; ++j) r[j] = 0u;
      }
      const int n = t * BM + row;
      const long long tu0 = (long long)t * kt;
      const int c_first = cta_of(tu0, U, G);
      const int nc = cta_of(tu0 + kt - 1, U, G) - c_first + 1;
      bool complete = false;
      if (nc == 1) {
        for (int m = 0; m < g.M; ++m)
          write_value<PUSH>(g, push, seq, m, n, lane, __uint_as_float(r[m]) * g.a_scale[m]);
        complete = true;
      } else {
        // my partial -> my slot (first segment of my range: slot 2c, last: 2c + 1)
        float* slot = g.part + ((size_t)(2 * c + (seg == 0 ? 0 : 1)) * BN) * BM;
        for (int m = 0; m < g.M; ++m) slot[m * BM + row] = __uint_as_float(r[m]);
        __threadfence();
        asm volatile("bar.sync 3, 128;" ::: "memory");
        if (threadIdx.x == 64) {
          const unsigned old = atomicAdd(&g.tile_cnt[t], 1u);
          s_last = old == (unsigned)(nc - 1);
          if (s_last) g.tile_cnt[t] = 0u;
        }
        asm volatile("bar.sync 3, 128;" ::: "memory");
        if (s_last) {
          __threadfence();
          for (int m = 0; m < g.M; ++m) {
            float acc = 0.f;
            for (int j = 0; j < nc; ++j) {
              const int cc = c_first + j;
              const int sl = 2 * cc + (range_lo(cc, U, G) < tu0 ? 1 : 0);
              acc += __ldcg(g.part + ((size_t)sl * BN + m) * BM + row);
            }
            write_value<PUSH>(g, push, seq, m, n, lane, acc * g.a_scale[m]);
          }
          complete = true;
        }
      }
      if (FIN != kFinNone && complete) {
        __threadfence();
        asm volatile("bar.sync 3, 128;" ::: "memory");
        if (threadIdx.x == 64) {
          const unsigned old = atomicAdd(g.done_cnt, 1u);
          if (old == (unsigned)(g.tiles - 1)) {
            s_fin = 1;
            *g.done_cnt = 0u;
          }
        }
      }
      i += len;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
  if constexpr (FIN != kFinNone) {
    if (s_fin) {   // every output tile is written: finish the row(s) with all six warps
      __threadfence();
      float* buf = reinterpret_cast<float*>(stage_base);
      for (int m = 0; m < g.M; ++m) finish_row<kThreads, FIN>(fin, g.out, g.ldo, g.N, m, buf, s_red);
    }
  }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
struct MapKey {
  uintptr_t ptr;
  int64_t rows, cols, stride;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && rows == o.rows && cols == o.cols && stride == o.stride;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<uintptr_t>()(k.ptr) ^ (std::hash<int64_t>()(k.rows) << 1) ^
           (std::hash<int64_t>()(k.cols) << 7);
  }
};
static std::mutex g_mu;
static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_wmaps;

static CUtensorMap weight_map(const torch::Tensor& packed, int64_t N, int64_t K) {
  MapKey key{(uintptr_t)packed.data_ptr(), N, K, packed.stride(0)};
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_wmaps.find(key);
  if (it != g_wmaps.end()) return it->second;
  CUtensorMap m = make_tma_2d(packed.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, K, N,
                              packed.stride(0), BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  g_wmaps.emplace(key, m);
  return m;
}

static int num_sms() {
  static int n = [] {
    int dev = 0, v = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
      cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
  }();
  return n;
}

static int64_t launch(const torch::Tensor& a, const torch::Tensor& a_scale, const torch::Tensor& wp,
                      const torch::Tensor& sf, const torch::Tensor& out, const torch::Tensor& ws,
                      int ctas_per_sm, const PushArgs& push, int fin_mode, const FinArgs& fa,
                      int* status) {
  const int M = a.size(0), K = a.size(1), N = wp.size(0);
  const int Kw = (int)wp.size(1) * 2;
  TORCH_CHECK(a.scalar_type() == at::kFloat8_e4m3fn, "mxfp4_gemv: e4m3 activations");
  TORCH_CHECK(M >= 1 && M <= BN, "mxfp4_gemv: 1..16 activation rows");
  TORCH_CHECK(a.stride(1) == 1 && (a.stride(0) % 16) == 0 &&
                  (reinterpret_cast<uintptr_t>(a.data_ptr()) % 16) == 0,
              "mxfp4_gemv: activation rows 16-byte aligned");
  TORCH_CHECK(K % 32 == 0 && Kw % BK == 0 && Kw >= K && Kw - K < BK,
              "mxfp4_gemv: weight K must be the activation K rounded up to a multiple of 128");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(wp.data_ptr()) % 32) == 0 && (wp.stride(0) % 32) == 0,
              "mxfp4_gemv: weight rows 32-byte aligned");
  const int kt = Kw / BK;
  const int tiles = (N + BM - 1) / BM;
  TORCH_CHECK(tiles <= kTileCounters, "mxfp4_gemv: at most 4096 output tiles");
  const long long units = (long long)tiles * kt;
  int G = (int)std::min<long long>(units, (long long)num_sms() * std::max(1, ctas_per_sm));
  TORCH_CHECK(ws.scalar_type() == at::kInt && ws.numel() >= kPartOff + (int64_t)2 * G * BN * BM,
              "mxfp4_gemv: workspace too small");
  if (fin_mode != kFinNone) {
    TORCH_CHECK(!push.world, "mxfp4_gemv: a finisher needs a local output");
    TORCH_CHECK(N % 8 == 0 && (fin_mode == kFinNorm ? N : N / 2) <= kMaxFinH &&
                    (fin_mode == kFinNorm || N % 16 == 0),
                "mxfp4_gemv: finisher row length");
    TORCH_CHECK(out.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(out.data_ptr()) % 16) == 0,
                "mxfp4_gemv: finisher reads 16-byte aligned output rows");
  }
  const at::cuda::CUDAGuard guard(a.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  CUtensorMap tw = weight_map(wp, N, Kw);
  CUtensorMap ta = make_tma_2d(a.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, K, M, a.stride(0), BK,
                               BN, CU_TENSOR_MAP_SWIZZLE_128B);
  GemvArgs ga{};
  ga.sfw = (const uint8_t*)sf.data_ptr();
  ga.a_scale = a_scale.data_ptr<float>();
  ga.out = push.world ? nullptr : (__nv_bfloat16*)out.data_ptr();
  ga.ldo = push.world ? 0 : (int)out.stride(0);
  ga.M = M;
  ga.N = N;
  ga.kt = kt;
  ga.tiles = tiles;
  ga.units = units;
  unsigned* wsu = reinterpret_cast<unsigned*>(ws.data_ptr());
  ga.tile_cnt = wsu;
  ga.done_cnt = wsu + kDoneOff;
  ga.part = reinterpret_cast<float*>(ws.data_ptr<int>() + kPartOff);
  ga.status = status;
  using KernT = decltype(&gemv_kernel<false, kFinNone>);
  KernT kern;
  int variant;
  if (push.world) { kern = gemv_kernel<true, kFinNone>; variant = 1; }
  else if (fin_mode == kFinNorm) { kern = gemv_kernel<false, kFinNorm>; variant = 2; }
  else if (fin_mode == kFinSilu) { kern = gemv_kernel<false, kFinSilu>; variant = 3; }
  else { kern = gemv_kernel<false, kFinNone>; variant = 0; }
  static bool attr_set[4] = {false, false, false, false};
  if (!attr_set[variant]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    attr_set[variant] = true;
  }
  C10_CUDA_CHECK(launch_pdl(kern, dim3(G), dim3(kThreads), SMEM_BYTES, stream, tw, ta, ga, push, fa));
  return tiles;
}

static const __nv_bfloat16* bfp(const torch::Tensor& t) {
  return t.defined() && t.numel() ? reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()) : nullptr;
}

}  // namespace gemv

// Decode GEMM (1..16 rows): out [M, N] bf16.  fin_mode 0: out only; 1: out, then residual add +
// RMSNorm(1 + w) + e4m3 of each out row (res optional, res_out optional, q [M, N], scale [M]);
// 2: out = [g | u], then SiLU(g) * u + e4m3 (q [M, N/2]).  ws: int32 workspace (zero-initialised,
// >= 8192 + 2 * 148 * ctas_per_sm * 2048 elements; its counters are self-resetting).
void mxfp4_gemv(torch::Tensor a, torch::Tensor a_scale, torch::Tensor wp, torch::Tensor sf,
                torch::Tensor out, torch::Tensor ws, int64_t ctas_per_sm, int64_t fin_mode,
                torch::Tensor res, torch::Tensor w, torch::Tensor res_out, torch::Tensor q,
                torch::Tensor scale, double eps, torch::Tensor status) {
  using namespace gemv;
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(1) == 1 && out.size(0) >= a.size(0) &&
                  out.size(1) >= wp.size(0), "mxfp4_gemv: out");
  FinArgs fa{};
  if (fin_mode != kFinNone) {
    const int M = a.size(0), N = wp.size(0);
    const int H = fin_mode == kFinNorm ? N : N / 2;
    TORCH_CHECK(q.defined() && q.scalar_type() == at::kFloat8_e4m3fn && q.size(0) >= M &&
                    q.size(1) >= H && q.stride(1) == 1 && q.stride(0) % 8 == 0, "mxfp4_gemv: q");
    TORCH_CHECK(scale.defined() && scale.scalar_type() == at::kFloat && scale.numel() >= M, "scale");
    fa.q = (uint8_t*)q.data_ptr();
    fa.ldq = (int)q.stride(0);
    fa.scale = scale.data_ptr<float>();
    fa.eps = (float)eps;
    if (fin_mode == kFinNorm) {
      TORCH_CHECK(w.defined() && w.numel() >= N && w.scalar_type() == at::kBFloat16, "norm weight");
      fa.w = bfp(w);
      fa.res = bfp(res);
      fa.ldr = fa.res ? (int)res.stride(0) : 0;
      fa.res_out = res_out.defined() && res_out.numel() ? (__nv_bfloat16*)res_out.data_ptr() : nullptr;
      fa.ldro = fa.res_out ? (int)res_out.stride(0) : 0;
      TORCH_CHECK(!fa.res || (res.stride(1) == 1 && res.stride(0) % 8 == 0), "res rows");
      TORCH_CHECK(!fa.res_out || (res_out.stride(1) == 1 && res_out.stride(0) % 8 == 0), "res_out rows");
    }
  }
  int* st = status.numel() ? status.data_ptr<int>() : nullptr;
  launch(a, a_scale, wp, sf, out, ws, (int)ctas_per_sm, PushArgs{}, (int)fin_mode, fa, st);
}

// Row-parallel decode GEMM fused with the push half of the all-reduce (see mxfp4_gemm_push):
// the output tiles go to every rank's receive buffer instead of a local tensor.
int64_t mxfp4_gemv_push(torch::Tensor a, torch::Tensor a_scale, torch::Tensor wp, torch::Tensor sf,
                        torch::Tensor ws, int64_t ctas_per_sm, std::vector<int64_t> peers,
                        int64_t rank, int64_t half_words, torch::Tensor status) {
  using namespace gemv;
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
  int* st = status.numel() ? status.data_ptr<int>() : nullptr;
  return launch(a, a_scale, wp, sf, torch::Tensor(), ws, (int)ctas_per_sm, pa, kFinNone, FinArgs{}, st);
}

}  // namespace rad
