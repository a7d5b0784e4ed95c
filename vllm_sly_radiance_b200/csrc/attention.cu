// Paged attention for the hybrid model's full-attention layers (head_dim 64 or 256, GQA, fp8 or
// bf16 KV cache in pages of 64 tokens, layout [block, kv_head, slot, head_dim]).
//
// Reference behaviour: the AITER unified attention the reference tunes for decode/verify
// (sly/radiance_attn_decode.py:115-209: split-KV with segment reduce) and the libr4d paged prefill
// kernel (r4d_attn_prefill_h256_gqa6, radiance_r4d_hybrid_attn.py:1-97: chunked causal prefill
// over the paged fp8 cache, e4m3 query).  Here one varlen kernel serves both:
//
//  * qkv_prologue : per (token, head) Gemma RMSNorm of q and k, neox RoPE on the first rotary_dim
//                   dims (cos/sin table precomputed in fp64), k and v written to the paged cache
//                   (e4m3), q written as bf16 (rounded through e4m3 when the cache is fp8, the
//                   reference's fp8-query contract).
//  * paged_attn   : rows = (query token, q head of the GQA group) of one kv head, 64 rows per CTA
//                   (4 warps x 16), keys in 64-token pages; S = QK^T and O += PV on tensor cores,
//                   online softmax in registers, causal + sliding-window masks.  Split-KV along the
//                   context with a per-sequence split length computed on the device (CUDA-graph
//                   safe); partials merged by attn_merge.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cuda_fp16.h>

#include "common.cuh"

namespace rad {
namespace attn {

// ------------------------------------------------------------------------------------------------
// prologue: one warp per (token, head); heads [0, Hq) are q heads, [Hq, Hq+Hkv) kv heads
// ------------------------------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256) qkv_prologue_kernel(
    const __nv_bfloat16* __restrict__ qkv, int ldqkv, int q_head_stride,   // q head h at col h*q_head_stride
    int k_off, int v_off, const int* __restrict__ positions,
    const __nv_bfloat16* __restrict__ qn_w, const __nv_bfloat16* __restrict__ kn_w,
    const float* __restrict__ cos_sin, int rot, int T, int Hq, int Hkv, float eps,
    __nv_bfloat16* __restrict__ q_out, uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache,
    int cache_fmt, const int64_t* __restrict__ slot_mapping, int block_size) {
  // cache_fmt: 0 bf16, 1 fp8 e4m3, 2 int4 (+ fp16 scale/zero per 16 elements)
  const int cache_fp8 = cache_fmt == 1;
  constexpr int PER = D / 32;
  const int gw = blockIdx.x * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int H = Hq + Hkv;
  const int t = gw / H, h = gw % H;
  const bool isq = h < Hq;
  // the RMSNorm weight is a model constant: fetched before the dependency wait
  float nwv[PER];
  {
    const __nv_bfloat16* nw = isq ? qn_w : kn_w;
#pragma unroll
    for (int p = 0; p < PER; ++p) nwv[p] = __bfloat162float(nw[lane * PER + p]);
  }
  pdl_wait();     // inputs come from the preceding kernel
  pdl_trigger();
  if (gw >= T * H) return;
  const __nv_bfloat16* src = qkv + (size_t)t * ldqkv + (isq ? h * q_head_stride : k_off + (h - Hq) * D);
  float x[PER];
  float ss = 0.f;
#pragma unroll
  for (int p = 0; p < PER; ++p) {
    x[p] = __bfloat162float(src[lane * PER + p]);
    ss += x[p] * x[p];
  }
  ss = warp_sum(ss);
  const float rs = rsqrtf(ss / (float)D + eps);
#pragma unroll
  for (int p = 0; p < PER; ++p) x[p] = bf16_round(x[p] * rs * (nwv[p] + 1.f));
  // RoPE (neox): element i < rot/2 pairs with i + rot/2
  const int pos = positions[t];
  const int half = rot / 2;
  const int off = half / PER;            // partner lane distance (power of two)
  float partner[PER];
#pragma unroll
  for (int p = 0; p < PER; ++p) partner[p] = __shfl_xor_sync(0xffffffff, x[p], off > 0 ? off : 1);
  if (lane * PER < rot) {
#pragma unroll
    for (int p = 0; p < PER; ++p) {
      const int i = lane * PER + p;
      const int fi = i % half;
      const float c = cos_sin[(size_t)pos * rot + fi];
      const float s = cos_sin[(size_t)pos * rot + half + fi];
      x[p] = (i < half) ? (x[p] * c - partner[p] * s) : (x[p] * c + partner[p] * s);
    }
  }
  if (isq) {
    __nv_bfloat16* dst = q_out + ((size_t)t * Hq + h) * D;
#pragma unroll
    for (int p = 0; p < PER; ++p) {
      float v = bf16_round(x[p]);
      if (cache_fmt == 1) v = e4m3_to_f32(f32_to_e4m3(v));
      dst[lane * PER + p] = __float2bfloat16_rn(v);
    }
  } else {
    const int hk = h - Hq;
    const int64_t slot = slot_mapping[t];
    if (slot < 0) return;
    const int64_t blk = slot / block_size, off2 = slot % block_size;
    const __nv_bfloat16* vsrc = qkv + (size_t)t * ldqkv + v_off + hk * D;
    if (cache_fmt == 2) {
      // 4-bit rows: [D/2 nibble bytes][D/16 x (fp16 scale, fp16 zero)]
      constexpr int RB = D / 2 + D / 4;
      constexpr int LPG = 16 / PER;                 // lanes per 16-element group
      const size_t row = (((size_t)blk * Hkv + hk) * block_size + off2) * RB;
      float vv[PER];
#pragma unroll
      for (int p = 0; p < PER; ++p) vv[p] = __bfloat162float(vsrc[lane * PER + p]);
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        float* xs = which == 0 ? x : vv;
        uint8_t* dst = (which == 0 ? k_cache : v_cache) + row;
        float lo = 1e30f, hi = -1e30f;
#pragma unroll
        for (int p = 0; p < PER; ++p) {
          const float e = which == 0 ? bf16_round(xs[p]) : xs[p];
          lo = fminf(lo, e);
          hi = fmaxf(hi, e);
        }
#pragma unroll
        for (int o = 1; o < LPG; o <<= 1) {
          lo = fminf(lo, __shfl_xor_sync(0xffffffff, lo, o));
          hi = fmaxf(hi, __shfl_xor_sync(0xffffffff, hi, o));
        }
        float sc = (hi - lo) / 15.f;
        if (!(sc > 0.f)) sc = 1.f;
        const __half sc16 = __float2half_rn(sc), lo16 = __float2half_rn(lo);
        const float scf = __half2float(sc16), lof = __half2float(lo16);
        uint32_t packed = 0;
#pragma unroll
        for (int p = 0; p < PER; ++p) {
          const float e = which == 0 ? bf16_round(xs[p]) : xs[p];
          const int qv = min(15, max(0, __float2int_rn((e - lof) / scf)));
          packed |= (uint32_t)qv << (4 * p);
        }
#pragma unroll
        for (int b = 0; b < PER / 2; ++b) dst[lane * PER / 2 + b] = (uint8_t)(packed >> (8 * b));
        if ((lane % LPG) == 0) {
          const int gi = lane / LPG;
          __half2 m = __halves2half2(sc16, lo16);
          *reinterpret_cast<__half2*>(dst + D / 2 + gi * 4) = m;
        }
      }
      return;
    }
    const size_t base = (((size_t)blk * Hkv + hk) * block_size + off2) * D;
    if (cache_fp8) {
#pragma unroll
      for (int p = 0; p < PER; ++p) {
        k_cache[base + lane * PER + p] = f32_to_e4m3(bf16_round(x[p]));
        v_cache[base + lane * PER + p] = f32_to_e4m3(__bfloat162float(vsrc[lane * PER + p]));
      }
    } else {
      __nv_bfloat16* kc = reinterpret_cast<__nv_bfloat16*>(k_cache);
      __nv_bfloat16* vc = reinterpret_cast<__nv_bfloat16*>(v_cache);
#pragma unroll
      for (int p = 0; p < PER; ++p) {
        kc[base + lane * PER + p] = __float2bfloat16_rn(x[p]);
        vc[base + lane * PER + p] = vsrc[lane * PER + p];
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------
// paged attention
// ------------------------------------------------------------------------------------------------
constexpr int BR = 64;        // rows per CTA
constexpr int BC = 64;        // keys per tile (= one KV page)

DEVI void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
DEVI void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
DEVI void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                   uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
DEVI uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
// swizzled byte offset of (row, 16-byte chunk) in a tile with `chunks` chunks per row
DEVI uint32_t swz(int row, int chunk, int chunks) { return (uint32_t)(row * chunks + (chunk ^ (row & 7))) * 16u; }

template <int D, int FMT>
__global__ void __launch_bounds__(128) paged_attn_kernel(
    const __nv_bfloat16* __restrict__ q, const uint8_t* __restrict__ k_cache,
    const uint8_t* __restrict__ v_cache, const int* __restrict__ block_tables, int bt_stride,
    const int* __restrict__ seq_lens, const int* __restrict__ qsl,
    const int* __restrict__ tile_seq, const int* __restrict__ tile_row0, int Hq, int Hkv,
    int block_size, float scale_log2, int causal, int window, int num_splits,
    __nv_bfloat16* __restrict__ out, float* __restrict__ part_o, float* __restrict__ part_ml,
    int T, unsigned* __restrict__ counters) {
  pdl_wait();     // inputs come from the preceding kernel
  pdl_trigger();
  __shared__ bool s_last;
  constexpr int CH = D / 8;               // 16-byte chunks per row (bf16)
  constexpr int NT = BC / 8;              // n-tiles of S per warp (8 keys each)
  constexpr int OT = D / 8;               // n-tiles of O per warp
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;                                   // [BR][D] bf16 swizzled
  uint8_t* sK = smem + BR * D * 2;                      // [BC][D]
  uint8_t* sV = sK + BC * D * 2;                        // [BC][D]

  const int tile = blockIdx.x, hk = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int b = tile_seq[tile];
  const int row0 = tile_row0[tile];
  const int G = Hq / Hkv;
  const int s0 = qsl[b];
  const int ql = qsl[b + 1] - s0;
  const int L = seq_lens[b];
  const int R = ql * G;
  const int rows_here = min(BR, R - row0);
  // key range needed by this tile: causal -> up to the last row's position
  const int last_i = (row0 + rows_here - 1) / G;
  const int first_i = row0 / G;
  const int kv_end = causal ? (L - ql + last_i + 1) : L;
  int kv_begin = 0;
  if (window > 0) kv_begin = max(0, L - ql + first_i - window + 1);
  // split range (device-side, graph safe)
  const int ntiles_total = (kv_end + BC - 1) / BC;
  const int tile_begin = kv_begin / BC;
  const int ntiles = ntiles_total - tile_begin;
  const int per = (ntiles + num_splits - 1) / num_splits;
  const int t_lo = tile_begin + split * per;
  const int t_hi = min(ntiles_total, t_lo + per);

  // ---- load Q tile (rows beyond R zero) ----
  for (int idx = threadIdx.x; idx < BR * CH; idx += 128) {
    const int r = idx / CH, c = idx % CH;
    uint4 val = make_uint4(0, 0, 0, 0);
    const int rr = row0 + r;
    if (rr < R) {
      const int i = rr / G, g = rr % G;
      const __nv_bfloat16* src = q + ((size_t)(s0 + i) * Hq + hk * G + g) * D + c * 8;
      val = *reinterpret_cast<const uint4*>(src);
    }
    *reinterpret_cast<uint4*>(sQ + swz(r, c, CH)) = val;
  }

  float o[OT][4];
#pragma unroll
  for (int j = 0; j < OT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const int g_ = lane / 4, t4 = lane % 4;
  // query positions of this thread's two rows
  const int rA = row0 + warp * 16 + g_, rB = rA + 8;
  const int posA = L - ql + rA / G, posB = L - ql + rB / G;
  const uint32_t sQa = smem_u32(sQ), sKa = smem_u32(sK), sVa = smem_u32(sV);

  for (int kt = t_lo; kt < t_hi; ++kt) {
    __syncthreads();
    // ---- load K/V tile kt (64 keys; pages of block_size tokens, any size dividing 64 or a
    //      multiple of 64), converting fp8 / int4 to bf16 in shared memory ----
    const int key0 = kt * BC;
    if constexpr (FMT == 1) {
      // all of this thread's 16-byte loads of the tile are issued before the first conversion, so
      // a tile costs about one memory latency instead of one per chunk
      constexpr int IT = BC * D / 16 / 128;
      uint4 kraw[IT], vraw[IT];
#pragma unroll
      for (int it = 0; it < IT; ++it) {
        const int idx = threadIdx.x + it * 128;
        const int r = idx / (D / 16), c16 = idx % (D / 16);
        const int key = key0 + r;
        kraw[it] = make_uint4(0, 0, 0, 0);
        vraw[it] = make_uint4(0, 0, 0, 0);
        if (key < L) {
          const int blk = block_tables[(size_t)b * bt_stride + key / block_size];
          const size_t base = (((size_t)blk * Hkv + hk) * block_size + key % block_size) * D;
          kraw[it] = __ldg(reinterpret_cast<const uint4*>(k_cache + base + c16 * 16));
          vraw[it] = __ldg(reinterpret_cast<const uint4*>(v_cache + base + c16 * 16));
        }
      }
#pragma unroll
      for (int it = 0; it < IT; ++it) {
        const int idx = threadIdx.x + it * 128;
        const int r = idx / (D / 16), c16 = idx % (D / 16);   // 16 fp8 = two bf16 chunks
        const uint8_t* kb = reinterpret_cast<const uint8_t*>(&kraw[it]);
        const uint8_t* vb = reinterpret_cast<const uint8_t*>(&vraw[it]);
        uint32_t kw[8], vw[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          kw[e] = pack_bf16(e4m3_to_f32(kb[2 * e]), e4m3_to_f32(kb[2 * e + 1]));
          vw[e] = pack_bf16(e4m3_to_f32(vb[2 * e]), e4m3_to_f32(vb[2 * e + 1]));
        }
        *reinterpret_cast<uint4*>(sK + swz(r, 2 * c16, CH)) = make_uint4(kw[0], kw[1], kw[2], kw[3]);
        *reinterpret_cast<uint4*>(sK + swz(r, 2 * c16 + 1, CH)) = make_uint4(kw[4], kw[5], kw[6], kw[7]);
        *reinterpret_cast<uint4*>(sV + swz(r, 2 * c16, CH)) = make_uint4(vw[0], vw[1], vw[2], vw[3]);
        *reinterpret_cast<uint4*>(sV + swz(r, 2 * c16 + 1, CH)) = make_uint4(vw[4], vw[5], vw[6], vw[7]);
      }
    } else if constexpr (FMT == 2) {
      constexpr int RB = D / 2 + D / 4;
      constexpr int IT = BC * D / 16 / 128;
      // raw loads of the whole tile first (nibbles + (scale, zero) per 16-element group)
      uint2 knib[IT], vnib[IT];
      __half2 kmz[IT], vmz[IT];
#pragma unroll
      for (int it = 0; it < IT; ++it) {
        const int idx = threadIdx.x + it * 128;
        const int r = idx / (D / 16), g = idx % (D / 16);
        const int key = key0 + r;
        knib[it] = vnib[it] = make_uint2(0, 0);
        kmz[it] = vmz[it] = __floats2half2_rn(0.f, 0.f);
        if (key < L) {
          const int blk = block_tables[(size_t)b * bt_stride + key / block_size];
          const size_t row = (((size_t)blk * Hkv + hk) * block_size + key % block_size) * RB;
          knib[it] = __ldg(reinterpret_cast<const uint2*>(k_cache + row + g * 8));
          vnib[it] = __ldg(reinterpret_cast<const uint2*>(v_cache + row + g * 8));
          kmz[it] = *reinterpret_cast<const __half2*>(k_cache + row + D / 2 + g * 4);
          vmz[it] = *reinterpret_cast<const __half2*>(v_cache + row + D / 2 + g * 4);
        }
      }
#pragma unroll
      for (int it = 0; it < IT; ++it) {
        const int idx = threadIdx.x + it * 128;
        const int r = idx / (D / 16), g = idx % (D / 16);     // one 16-element group
        uint32_t kw[8], vw[8];
#pragma unroll
        for (int which = 0; which < 2; ++which) {
          const uint2 nib = which == 0 ? knib[it] : vnib[it];
          const __half2 m = which == 0 ? kmz[it] : vmz[it];
          const float sc = __low2float(m), zr = __high2float(m);
          uint32_t* w = which == 0 ? kw : vw;
          const uint32_t lo32 = nib.x, hi32 = nib.y;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const uint32_t word = e < 4 ? lo32 : hi32;
            const int sh = (e % 4) * 8;
            const float a = (float)((word >> sh) & 0xF) * sc + zr;
            const float c = (float)((word >> (sh + 4)) & 0xF) * sc + zr;
            w[e] = pack_bf16(a, c);
          }
        }
        *reinterpret_cast<uint4*>(sK + swz(r, 2 * g, CH)) = make_uint4(kw[0], kw[1], kw[2], kw[3]);
        *reinterpret_cast<uint4*>(sK + swz(r, 2 * g + 1, CH)) = make_uint4(kw[4], kw[5], kw[6], kw[7]);
        *reinterpret_cast<uint4*>(sV + swz(r, 2 * g, CH)) = make_uint4(vw[0], vw[1], vw[2], vw[3]);
        *reinterpret_cast<uint4*>(sV + swz(r, 2 * g + 1, CH)) = make_uint4(vw[4], vw[5], vw[6], vw[7]);
      }
    } else {
      const __nv_bfloat16* kc = reinterpret_cast<const __nv_bfloat16*>(k_cache);
      const __nv_bfloat16* vc = reinterpret_cast<const __nv_bfloat16*>(v_cache);
      // loads issued in batches of up to 8 chunks per thread before the shared-memory stores
      constexpr int IT = BC * CH / 128;
      constexpr int BATCH = IT < 8 ? IT : 8;
#pragma unroll
      for (int it0 = 0; it0 < IT; it0 += BATCH) {
        uint4 kx[BATCH], vx[BATCH];
#pragma unroll
        for (int u = 0; u < BATCH; ++u) {
          const int idx = threadIdx.x + (it0 + u) * 128;
          const int r = idx / CH, c = idx % CH;
          const int key = key0 + r;
          kx[u] = make_uint4(0, 0, 0, 0);
          vx[u] = make_uint4(0, 0, 0, 0);
          if (key < L) {
            const int blk = block_tables[(size_t)b * bt_stride + key / block_size];
            const size_t base = (((size_t)blk * Hkv + hk) * block_size + key % block_size) * D;
            kx[u] = __ldg(reinterpret_cast<const uint4*>(kc + base + c * 8));
            vx[u] = __ldg(reinterpret_cast<const uint4*>(vc + base + c * 8));
          }
        }
#pragma unroll
        for (int u = 0; u < BATCH; ++u) {
          const int idx = threadIdx.x + (it0 + u) * 128;
          const int r = idx / CH, c = idx % CH;
          *reinterpret_cast<uint4*>(sK + swz(r, c, CH)) = kx[u];
          *reinterpret_cast<uint4*>(sV + swz(r, c, CH)) = vx[u];
        }
      }
    }
    __syncthreads();

    // warps whose 16 rows are all padding (decode: G rows per kv head) skip the math
    if (warp * 16 >= rows_here) continue;
    // ---- S = Q K^T (16 rows x 64 keys per warp) ----
    float s[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a0, a1, a2, a3;
      {
        const int r = warp * 16 + (lane % 16);
        const int c = kk * 2 + lane / 16;
        ldsm_x4(sQa + swz(r, c, CH), a0, a1, a2, a3);
      }
#pragma unroll
      for (int jn = 0; jn < NT; jn += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = jn * 8 + (lane % 8) + (lane / 16) * 8;
        const int c = kk * 2 + ((lane / 8) % 2);
        ldsm_x4(sKa + swz(r, c, CH), b0, b1, b2, b3);
        mma_bf16(s[jn], a0, a1, a2, a3, b0, b1);
        mma_bf16(s[jn + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    // ---- masks + online softmax ----
    const int k0 = kt * BC;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < NT; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = k0 + j * 8 + 2 * t4 + (e & 1);
        const int pos = (e < 2) ? posA : posB;
        bool ok = key < L;
        if (causal) ok = ok && key <= pos;
        if (window > 0) ok = ok && key > pos - window;
        const float v = ok ? s[j][e] * scale_log2 : -INFINITY;
        s[j][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffff, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffff, mx[h], 2));
    }
    float alpha[2], mnew[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mnew[h] = fmaxf(m_run[h], mx[h]);
      const float mref = mnew[h] == -INFINITY ? 0.f : mnew[h];
      alpha[h] = exp2f(m_run[h] - mref);
      m_run[h] = mnew[h];
    }
    float rsum[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < NT; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e >> 1;
        const float mref = mnew[h] == -INFINITY ? 0.f : mnew[h];
        const float p = exp2f(s[j][e] - mref);
        s[j][e] = p;
        rsum[h] += p;
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      rsum[h] += __shfl_xor_sync(0xffffffff, rsum[h], 1);
      rsum[h] += __shfl_xor_sync(0xffffffff, rsum[h], 2);
      l_run[h] = l_run[h] * alpha[h] + rsum[h];
    }
#pragma unroll
    for (int j = 0; j < OT; ++j) {
      o[j][0] *= alpha[0]; o[j][1] *= alpha[0];
      o[j][2] *= alpha[1]; o[j][3] *= alpha[1];
    }
    // ---- O += P V ----
#pragma unroll
    for (int kk = 0; kk < BC / 16; ++kk) {
      const uint32_t a0 = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      const uint32_t a1 = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t a2 = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t a3 = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int jn = 0; jn < OT; jn += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = kk * 16 + (lane % 8) + ((lane / 8) % 2) * 8;
        const int c = jn + lane / 16;
        ldsm_x4_t(sVa + swz(r, c, CH), b0, b1, b2, b3);
        mma_bf16(o[jn], a0, a1, a2, a3, b0, b1);
        mma_bf16(o[jn + 1], a0, a1, a2, a3, b2, b3);
      }
    }
  }

  // ---- epilogue ----
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int rr = (h == 0) ? rA : rB;
    if (rr >= R || rr - row0 >= BR) continue;
    const int i = rr / G, g = rr % G;
    const int tok = s0 + i, head = hk * G + g;
    const float inv = l_run[h] > 0.f ? 1.f / l_run[h] : 0.f;
    if (num_splits == 1) {
      __nv_bfloat16* dst = out + ((size_t)tok * Hq + head) * D;
#pragma unroll
      for (int j = 0; j < OT; ++j) {
        const int col = j * 8 + 2 * t4;
        *reinterpret_cast<__nv_bfloat162*>(dst + col) =
            __floats2bfloat162_rn(o[j][2 * h] * inv, o[j][2 * h + 1] * inv);
      }
    } else {
      float* dst = part_o + (((size_t)split * T + tok) * Hq + head) * D;
#pragma unroll
      for (int j = 0; j < OT; ++j) {
        const int col = j * 8 + 2 * t4;
        *reinterpret_cast<float2*>(dst + col) = make_float2(o[j][2 * h] * inv, o[j][2 * h + 1] * inv);
      }
      if (t4 == 0) {
        float* ml = part_ml + (((size_t)split * T + tok) * Hq + head) * 2;
        ml[0] = m_run[h];
        ml[1] = l_run[h];
      }
    }
  }
  if (num_splits > 1) {
    // the last split CTA of this (row tile, kv head) merges all splits' partials; every thread
    // fences its own partial stores before the arrival is counted
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      s_last = atomicAdd(&counters[tile * Hkv + hk], 1u) == (unsigned)(num_splits - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    constexpr int PER = D / 32;
    // splits past `used` had an empty key range; lane sp handles split sp's (m, l) (num_splits
    // <= 32 by construction of the host split count)
    const int used = per > 0 ? min(num_splits, (ntiles + per - 1) / per) : 1;
    for (int rr = warp; rr < rows_here; rr += 4) {
      const int r = row0 + rr;
      const int i = r / G, g = r % G;
      const size_t gw = (size_t)(s0 + i) * Hq + hk * G + g;
      float m = -INFINITY, l = 0.f;
      if (lane < used) {
        m = __ldcg(part_ml + ((size_t)lane * T * Hq + gw) * 2);
        l = __ldcg(part_ml + ((size_t)lane * T * Hq + gw) * 2 + 1);
      }
      float mmax = l > 0.f ? m : -INFINITY;
#pragma unroll
      for (int o2 = 16; o2 > 0; o2 >>= 1) mmax = fmaxf(mmax, __shfl_xor_sync(0xffffffff, mmax, o2));
      const float wl = l > 0.f ? l * exp2f(m - mmax) : 0.f;
      float wsum = wl;
#pragma unroll
      for (int o2 = 16; o2 > 0; o2 >>= 1) wsum += __shfl_xor_sync(0xffffffff, wsum, o2);
      float acc[PER];
#pragma unroll
      for (int p = 0; p < PER; ++p) acc[p] = 0.f;
      for (int sp0 = 0; sp0 < used; sp0 += 4) {
        float2 v[4][PER / 2];
        float w4[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int sp = sp0 + u;
          w4[u] = __shfl_sync(0xffffffff, wl, sp < used ? sp : 0);
          if (sp >= used) w4[u] = 0.f;
          const float2* src = reinterpret_cast<const float2*>(
              part_o + ((size_t)(sp < used ? sp : 0) * T * Hq + gw) * D + lane * PER);
#pragma unroll
          for (int p = 0; p < PER / 2; ++p) v[u][p] = w4[u] > 0.f ? __ldcg(src + p) : make_float2(0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int p = 0; p < PER / 2; ++p) {
            acc[2 * p + 0] += w4[u] * v[u][p].x;
            acc[2 * p + 1] += w4[u] * v[u][p].y;
          }
      }
      const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
#pragma unroll
      for (int p = 0; p < PER; ++p) out[gw * D + lane * PER + p] = __float2bfloat16_rn(acc[p] * inv);
    }
    if (threadIdx.x == 0) counters[tile * Hkv + hk] = 0;
  }
}


// ------------------------------------------------------------------------------------------------
// decode attention: at most 16 query rows per (sequence, kv head) -- one token's G query heads,
// or a short verify window when G * q_len <= 16.  The four warps split each 64-key tile's keys
// (16 each) instead of its rows, each keeps its own running (max, sum, O), and the CTA merges
// them in shared memory at the end.  With an fp8 cache, K/V convert to f16 with the hardware
// e4m3x2 -> f16x2 conversion and the MMAs run in f16 (exact: the query is e4m3-rounded when the
// cache is fp8, and e4m3 values are exact in f16); other formats use bf16 as the general kernel.
// ------------------------------------------------------------------------------------------------
DEVI void mma_f16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                  uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
DEVI uint32_t pack_f16(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
DEVI uint32_t e4m3x2_to_f16x2(uint16_t v) {
  __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)v, __NV_E4M3);
  return *reinterpret_cast<uint32_t*>(&h);
}

// The o_proj producer fused into decode attention (GQ): once the Hkv CTAs that write a token's
// heads are done (self-resetting per-token counter), the last one applies the sigmoid output
// gate to the token's row -- y = bf16(o / (1 + e^-gate)), the numerics of gate_mul_quant -- and
// quantises it to e4m3 with the per-token scale.  One token per tile (pure decode).
struct AttnGateArgs {
  const __nv_bfloat16* gate;    // gate of head h, column c: gate[tok * ldg + h * ghs + c]
  int ldg;
  int ghs;
  unsigned* tok_cnt;            // [T] arrival counters (zero, self-resetting)
  uint8_t* q;                   // [T, Hq * D] e4m3
  int ldq;
  float* q_scale;               // [T]
};

template <int D, int FMT, bool GQ = false>
__global__ void __launch_bounds__(128) paged_attn_decode_kernel(
    const __nv_bfloat16* __restrict__ q, const uint8_t* __restrict__ k_cache,
    const uint8_t* __restrict__ v_cache, const int* __restrict__ block_tables, int bt_stride,
    const int* __restrict__ seq_lens, const int* __restrict__ qsl,
    const int* __restrict__ tile_seq, const int* __restrict__ tile_row0, int Hq, int Hkv,
    int block_size, float scale_log2, int causal, int window, int num_splits,
    __nv_bfloat16* __restrict__ out, float* __restrict__ part_o, float* __restrict__ part_ml,
    int T, unsigned* __restrict__ counters, const AttnGateArgs ga) {
  pdl_wait();     // inputs come from the preceding kernel
  pdl_trigger();
  constexpr bool F16 = (FMT == 1);
  constexpr int QR = 16;                  // query rows per CTA
  constexpr int CH = D / 8;               // 16-byte chunks per row (16-bit elements)
  constexpr int OT = D / 8;
  __shared__ bool s_last;
  __shared__ float s_ml[4][QR][2];
  __shared__ float s_fin[QR][2];
  constexpr int MAXSP = 128;              // KV splits the in-kernel merge takes
  __shared__ float s_w[QR][MAXSP + 1];
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;                                   // [16][D]
  uint8_t* sK = smem + QR * D * 2;                      // [64][D]
  uint8_t* sV = sK + BC * D * 2;                        // [64][D]

  const int tile = blockIdx.x, hk = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int b = tile_seq[tile];
  const int row0 = tile_row0[tile];
  const int G = Hq / Hkv;
  const int s0 = qsl[b];
  const int ql = qsl[b + 1] - s0;
  const int L = seq_lens[b];
  const int R = ql * G;
  const int rows_here = min(QR, R - row0);
  const int last_i = (row0 + rows_here - 1) / G;
  const int first_i = row0 / G;
  const int kv_end = causal ? (L - ql + last_i + 1) : L;
  int kv_begin = 0;
  if (window > 0) kv_begin = max(0, L - ql + first_i - window + 1);
  const int ntiles_total = (kv_end + BC - 1) / BC;
  const int tile_begin = kv_begin / BC;
  const int ntiles = ntiles_total - tile_begin;
  const int per = (ntiles + num_splits - 1) / num_splits;
  const int t_lo = tile_begin + split * per;
  const int t_hi = min(ntiles_total, t_lo + per);

  // fp8 cache: the first tile's loads are issued before the query is staged, so both latencies
  // overlap
  constexpr int IT1 = BC * D / 16 / 128;
  uint4 kraw[IT1], vraw[IT1];
  auto load_raw = [&](int kt) {
#pragma unroll
    for (int it = 0; it < IT1; ++it) {
      const int idx = threadIdx.x + it * 128;
      const int r = idx / (D / 16), c16 = idx % (D / 16);
      const int key = kt * BC + r;
      kraw[it] = make_uint4(0, 0, 0, 0);
      vraw[it] = make_uint4(0, 0, 0, 0);
      if (key < L) {
        const int blk = block_tables[(size_t)b * bt_stride + key / block_size];
        const size_t base = (((size_t)blk * Hkv + hk) * block_size + key % block_size) * D;
        kraw[it] = __ldg(reinterpret_cast<const uint4*>(k_cache + base + c16 * 16));
        vraw[it] = __ldg(reinterpret_cast<const uint4*>(v_cache + base + c16 * 16));
      }
    }
  };
  if constexpr (FMT == 1) {
    if (t_lo < t_hi) load_raw(t_lo);
  }
  // int4 cache (4-bit codes + fp16 scale / zero per 16 elements): same one-tile-ahead prefetch
  constexpr int RB4 = D / 2 + D / 4;
  constexpr int IT4 = BC * D / 16 / 128;
  uint2 knib[FMT == 2 ? IT4 : 1], vnib[FMT == 2 ? IT4 : 1];
  __half2 kmz[FMT == 2 ? IT4 : 1], vmz[FMT == 2 ? IT4 : 1];
  auto load_nib = [&](int kt) {
    if constexpr (FMT == 2) {
#pragma unroll
      for (int it = 0; it < IT4; ++it) {
        const int idx = threadIdx.x + it * 128;
        const int r = idx / (D / 16), g = idx % (D / 16);
        const int key = kt * BC + r;
        knib[it] = vnib[it] = make_uint2(0, 0);
        kmz[it] = vmz[it] = __floats2half2_rn(0.f, 0.f);
        if (key < L) {
          const int blk = block_tables[(size_t)b * bt_stride + key / block_size];
          const size_t row = (((size_t)blk * Hkv + hk) * block_size + key % block_size) * RB4;
          knib[it] = __ldg(reinterpret_cast<const uint2*>(k_cache + row + g * 8));
          vnib[it] = __ldg(reinterpret_cast<const uint2*>(v_cache + row + g * 8));
          kmz[it] = *reinterpret_cast<const __half2*>(k_cache + row + D / 2 + g * 4);
          vmz[it] = *reinterpret_cast<const __half2*>(v_cache + row + D / 2 + g * 4);
        }
      }
    }
  };
  if constexpr (FMT == 2) {
    if (t_lo < t_hi) load_nib(t_lo);
  }

  // ---- Q (16 rows; rows past R are zero) ----
  for (int idx = threadIdx.x; idx < QR * CH; idx += 128) {
    const int r = idx / CH, c = idx % CH;
    uint4 val = make_uint4(0, 0, 0, 0);
    const int rr = row0 + r;
    if (r < rows_here) {
      const int i = rr / G, g = rr % G;
      val = *reinterpret_cast<const uint4*>(q + ((size_t)(s0 + i) * Hq + hk * G + g) * D + c * 8);
      if constexpr (F16) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&val);
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          w[e] = pack_f16(f.x, f.y);
        }
        val = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    *reinterpret_cast<uint4*>(sQ + swz(r, c, CH)) = val;
  }

  float o[OT][4];
#pragma unroll
  for (int j = 0; j < OT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const int g_ = lane / 4, t4 = lane % 4;
  const int rA = row0 + g_, rB = rA + 8;
  const int posA = L - ql + rA / G, posB = L - ql + rB / G;
  const uint32_t sQa = smem_u32(sQ), sKa = smem_u32(sK), sVa = smem_u32(sV);
  const int kw0 = warp * 16;              // this warp's keys within the tile

  for (int kt = t_lo; kt < t_hi; ++kt) {
    __syncthreads();
    const int key0 = kt * BC;
    if constexpr (FMT == 1) {
      constexpr int IT = IT1;
#pragma unroll
      for (int it = 0; it < IT; ++it) {
        const int idx = threadIdx.x + it * 128;
        const int r = idx / (D / 16), c16 = idx % (D / 16);
        const uint16_t* kb = reinterpret_cast<const uint16_t*>(&kraw[it]);
        const uint16_t* vb = reinterpret_cast<const uint16_t*>(&vraw[it]);
        uint32_t kw[8], vw[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          kw[e] = e4m3x2_to_f16x2(kb[e]);
          vw[e] = e4m3x2_to_f16x2(vb[e]);
        }
        *reinterpret_cast<uint4*>(sK + swz(r, 2 * c16, CH)) = make_uint4(kw[0], kw[1], kw[2], kw[3]);
        *reinterpret_cast<uint4*>(sK + swz(r, 2 * c16 + 1, CH)) = make_uint4(kw[4], kw[5], kw[6], kw[7]);
        *reinterpret_cast<uint4*>(sV + swz(r, 2 * c16, CH)) = make_uint4(vw[0], vw[1], vw[2], vw[3]);
        *reinterpret_cast<uint4*>(sV + swz(r, 2 * c16 + 1, CH)) = make_uint4(vw[4], vw[5], vw[6], vw[7]);
      }
      // the next tile's bytes travel while this tile's products run (one tile in flight ahead)
      if (kt + 1 < t_hi) load_raw(kt + 1);
    } else if constexpr (FMT == 2) {
      constexpr int IT = IT4;
#pragma unroll
      for (int it = 0; it < IT; ++it) {
        const int idx = threadIdx.x + it * 128;
        const int r = idx / (D / 16), g = idx % (D / 16);
        uint32_t kw[8], vw[8];
#pragma unroll
        for (int which = 0; which < 2; ++which) {
          const uint2 nib = which == 0 ? knib[it] : vnib[it];
          const __half2 m = which == 0 ? kmz[it] : vmz[it];
          const float sc = __low2float(m), zr = __high2float(m);
          uint32_t* w = which == 0 ? kw : vw;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const uint32_t word = e < 4 ? nib.x : nib.y;
            const int sh = (e % 4) * 8;
            w[e] = pack_bf16((float)((word >> sh) & 0xF) * sc + zr,
                             (float)((word >> (sh + 4)) & 0xF) * sc + zr);
          }
        }
        *reinterpret_cast<uint4*>(sK + swz(r, 2 * g, CH)) = make_uint4(kw[0], kw[1], kw[2], kw[3]);
        *reinterpret_cast<uint4*>(sK + swz(r, 2 * g + 1, CH)) = make_uint4(kw[4], kw[5], kw[6], kw[7]);
        *reinterpret_cast<uint4*>(sV + swz(r, 2 * g, CH)) = make_uint4(vw[0], vw[1], vw[2], vw[3]);
        *reinterpret_cast<uint4*>(sV + swz(r, 2 * g + 1, CH)) = make_uint4(vw[4], vw[5], vw[6], vw[7]);
      }
      if (kt + 1 < t_hi) load_nib(kt + 1);
    } else {
      const __nv_bfloat16* kc = reinterpret_cast<const __nv_bfloat16*>(k_cache);
      const __nv_bfloat16* vc = reinterpret_cast<const __nv_bfloat16*>(v_cache);
      constexpr int IT = BC * CH / 128;
      constexpr int BATCH = IT < 8 ? IT : 8;
#pragma unroll
      for (int it0 = 0; it0 < IT; it0 += BATCH) {
        uint4 kx[BATCH], vx[BATCH];
#pragma unroll
        for (int u = 0; u < BATCH; ++u) {
          const int idx = threadIdx.x + (it0 + u) * 128;
          const int r = idx / CH, c = idx % CH;
          const int key = key0 + r;
          kx[u] = make_uint4(0, 0, 0, 0);
          vx[u] = make_uint4(0, 0, 0, 0);
          if (key < L) {
            const int blk = block_tables[(size_t)b * bt_stride + key / block_size];
            const size_t base = (((size_t)blk * Hkv + hk) * block_size + key % block_size) * D;
            kx[u] = __ldg(reinterpret_cast<const uint4*>(kc + base + c * 8));
            vx[u] = __ldg(reinterpret_cast<const uint4*>(vc + base + c * 8));
          }
        }
#pragma unroll
        for (int u = 0; u < BATCH; ++u) {
          const int idx = threadIdx.x + (it0 + u) * 128;
          const int r = idx / CH, c = idx % CH;
          *reinterpret_cast<uint4*>(sK + swz(r, c, CH)) = kx[u];
          *reinterpret_cast<uint4*>(sV + swz(r, c, CH)) = vx[u];
        }
      }
    }
    __syncthreads();
    const int k0 = key0 + kw0;
    if (k0 >= kv_end) continue;           // this warp's 16 keys are all past the end

    // ---- S = Q K^T: 16 rows x this warp's 16 keys ----
    float sc[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
      ldsm_x4(sQa + swz(lane % 16, kk * 2 + lane / 16, CH), a0, a1, a2, a3);
      ldsm_x4(sKa + swz(kw0 + (lane % 8) + (lane / 16) * 8, kk * 2 + ((lane / 8) % 2), CH),
              b0, b1, b2, b3);
      if constexpr (F16) {
        mma_f16(sc[0], a0, a1, a2, a3, b0, b1);
        mma_f16(sc[1], a0, a1, a2, a3, b2, b3);
      } else {
        mma_bf16(sc[0], a0, a1, a2, a3, b0, b1);
        mma_bf16(sc[1], a0, a1, a2, a3, b2, b3);
      }
    }
    // ---- masks + online softmax (per warp) ----
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = k0 + j * 8 + 2 * t4 + (e & 1);
        const int pos = (e < 2) ? posA : posB;
        bool ok = key < L;
        if (causal) ok = ok && key <= pos;
        if (window > 0) ok = ok && key > pos - window;
        const float v = ok ? sc[j][e] * scale_log2 : -INFINITY;
        sc[j][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffff, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffff, mx[h], 2));
    }
    float alpha[2], mnew[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mnew[h] = fmaxf(m_run[h], mx[h]);
      const float mref = mnew[h] == -INFINITY ? 0.f : mnew[h];
      alpha[h] = exp2f(m_run[h] - mref);
      m_run[h] = mnew[h];
    }
    float rsum[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e >> 1;
        const float mref = mnew[h] == -INFINITY ? 0.f : mnew[h];
        const float p = exp2f(sc[j][e] - mref);
        sc[j][e] = p;
        rsum[h] += p;
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      rsum[h] += __shfl_xor_sync(0xffffffff, rsum[h], 1);
      rsum[h] += __shfl_xor_sync(0xffffffff, rsum[h], 2);
      l_run[h] = l_run[h] * alpha[h] + rsum[h];
    }
#pragma unroll
    for (int j = 0; j < OT; ++j) {
      o[j][0] *= alpha[0]; o[j][1] *= alpha[0];
      o[j][2] *= alpha[1]; o[j][3] *= alpha[1];
    }
    // ---- O += P V over this warp's 16 keys ----
    uint32_t a0, a1, a2, a3;
    if constexpr (F16) {
      a0 = pack_f16(sc[0][0], sc[0][1]); a1 = pack_f16(sc[0][2], sc[0][3]);
      a2 = pack_f16(sc[1][0], sc[1][1]); a3 = pack_f16(sc[1][2], sc[1][3]);
    } else {
      a0 = pack_bf16(sc[0][0], sc[0][1]); a1 = pack_bf16(sc[0][2], sc[0][3]);
      a2 = pack_bf16(sc[1][0], sc[1][1]); a3 = pack_bf16(sc[1][2], sc[1][3]);
    }
#pragma unroll
    for (int jn = 0; jn < OT; jn += 2) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(sVa + swz(kw0 + (lane % 8) + ((lane / 8) % 2) * 8, jn + lane / 16, CH), b0, b1, b2, b3);
      if constexpr (F16) {
        mma_f16(o[jn], a0, a1, a2, a3, b0, b1);
        mma_f16(o[jn + 1], a0, a1, a2, a3, b2, b3);
      } else {
        mma_bf16(o[jn], a0, a1, a2, a3, b0, b1);
        mma_bf16(o[jn + 1], a0, a1, a2, a3, b2, b3);
      }
    }
  }

  // ---- merge the four warps: M = max_w m_w, L = sum_w l_w 2^(m_w - M), O = sum_w o_w 2^(m_w - M)
  __syncthreads();                        // all warps are done with sK / sV
  float* sOw = reinterpret_cast<float*>(sK);            // [4][16][D] fp32 (fits sK + sV)
  if (t4 == 0) {
    s_ml[warp][g_][0] = m_run[0];
    s_ml[warp][g_][1] = l_run[0];
    s_ml[warp][g_ + 8][0] = m_run[1];
    s_ml[warp][g_ + 8][1] = l_run[1];
  }
  __syncthreads();
  float wself[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = g_ + 8 * h;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w)
      if (s_ml[w][r][1] > 0.f) M = fmaxf(M, s_ml[w][r][0]);
    wself[h] = (l_run[h] > 0.f) ? exp2f(m_run[h] - M) : 0.f;
    if (warp == 0 && t4 == 0) {
      float Ls = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w)
        if (s_ml[w][r][1] > 0.f) Ls += s_ml[w][r][1] * exp2f(s_ml[w][r][0] - M);
      s_fin[r][0] = M;
      s_fin[r][1] = Ls;
    }
  }
  float* myO = sOw + (size_t)warp * QR * D;
#pragma unroll
  for (int j = 0; j < OT; ++j) {
    const int col = j * 8 + 2 * t4;
    *reinterpret_cast<float2*>(myO + g_ * D + col) = make_float2(o[j][0] * wself[0], o[j][1] * wself[0]);
    *reinterpret_cast<float2*>(myO + (g_ + 8) * D + col) =
        make_float2(o[j][2] * wself[1], o[j][3] * wself[1]);
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < rows_here * (D / 4); idx += 128) {
    const int r = idx / (D / 4), c = (idx % (D / 4)) * 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float4 v = *reinterpret_cast<const float4*>(sOw + ((size_t)w * QR + r) * D + c);
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    const float Ls = s_fin[r][1];
    const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
    const int rr = row0 + r;
    const int i = rr / G, g = rr % G;
    const int tok = s0 + i, head = hk * G + g;
    if (num_splits == 1) {
      __nv_bfloat16* dst = out + ((size_t)tok * Hq + head) * D + c;
      *reinterpret_cast<__nv_bfloat162*>(dst) = __floats2bfloat162_rn(acc.x * inv, acc.y * inv);
      *reinterpret_cast<__nv_bfloat162*>(dst + 2) = __floats2bfloat162_rn(acc.z * inv, acc.w * inv);
    } else {
      *reinterpret_cast<float4*>(part_o + (((size_t)split * T + tok) * Hq + head) * D + c) =
          make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
      if (c == 0) {
        float* ml = part_ml + (((size_t)split * T + tok) * Hq + head) * 2;
        ml[0] = s_fin[r][0];
        ml[1] = Ls;
      }
    }
  }
  if (num_splits > 1) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      s_last = atomicAdd(&counters[tile * Hkv + hk], 1u) == (unsigned)(num_splits - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // splits past `used` had an empty key range (num_splits <= MAXSP by the host check)
    const int used = per > 0 ? min(num_splits, (ntiles + per - 1) / per) : 1;
    // weights per (row, split): warp w handles rows w, w + 4, ...; lane takes splits lane + 32 j
    for (int r = warp; r < rows_here; r += 4) {
      const int rr = row0 + r;
      const size_t gw = (size_t)(s0 + rr / G) * Hq + hk * G + rr % G;
      float mj[MAXSP / 32], lj[MAXSP / 32];
      float mmax = -INFINITY;
#pragma unroll
      for (int j = 0; j < MAXSP / 32; ++j) {
        const int sp = lane + 32 * j;
        mj[j] = -INFINITY;
        lj[j] = 0.f;
        if (sp < used) {
          mj[j] = __ldcg(part_ml + ((size_t)sp * T * Hq + gw) * 2);
          lj[j] = __ldcg(part_ml + ((size_t)sp * T * Hq + gw) * 2 + 1);
        }
        if (lj[j] > 0.f) mmax = fmaxf(mmax, mj[j]);
      }
#pragma unroll
      for (int o2 = 16; o2 > 0; o2 >>= 1) mmax = fmaxf(mmax, __shfl_xor_sync(0xffffffff, mmax, o2));
      float wsum = 0.f;
#pragma unroll
      for (int j = 0; j < MAXSP / 32; ++j) {
        const float wl = lj[j] > 0.f ? lj[j] * exp2f(mj[j] - mmax) : 0.f;
        wsum += wl;
        s_w[r][lane + 32 * j] = wl;
      }
#pragma unroll
      for (int o2 = 16; o2 > 0; o2 >>= 1) wsum += __shfl_xor_sync(0xffffffff, wsum, o2);
      if (lane == 0) s_w[r][MAXSP] = wsum;
    }
    __syncthreads();
    // 32 splits' partials of one 4-column group are loaded before any of them is summed
    for (int idx = threadIdx.x; idx < rows_here * (D / 4); idx += 128) {
      const int r = idx / (D / 4), c = (idx % (D / 4)) * 4;
      const int rr = row0 + r;
      const size_t gw = (size_t)(s0 + rr / G) * Hq + hk * G + rr % G;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int sp0 = 0; sp0 < used; sp0 += 32) {
        float4 v[32];
#pragma unroll
        for (int u = 0; u < 32; ++u)
          if (sp0 + u < used)
            v[u] = __ldcg(reinterpret_cast<const float4*>(part_o + ((size_t)(sp0 + u) * T * Hq + gw) * D + c));
#pragma unroll
        for (int u = 0; u < 32; ++u)
          if (sp0 + u < used) {
            const float w = s_w[r][sp0 + u];
            acc.x += w * v[u].x; acc.y += w * v[u].y; acc.z += w * v[u].z; acc.w += w * v[u].w;
          }
      }
      const float wsum = s_w[r][MAXSP];
      const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
      __nv_bfloat16* dst = out + gw * D + c;
      *reinterpret_cast<__nv_bfloat162*>(dst) = __floats2bfloat162_rn(acc.x * inv, acc.y * inv);
      *reinterpret_cast<__nv_bfloat162*>(dst + 2) = __floats2bfloat162_rn(acc.z * inv, acc.w * inv);
    }
    if (threadIdx.x == 0) counters[tile * Hkv + hk] = 0;
  }
  if constexpr (GQ) {
    // this CTA wrote the G heads of kv head hk for token s0 (one token per tile)
    const int tok = s0;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      s_last = atomicAdd(&ga.tok_cnt[tok], 1u) == (unsigned)(Hkv - 1);
      if (s_last) ga.tok_cnt[tok] = 0u;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // the token's whole row (Hq heads): gate, amax, e4m3
    float* buf = reinterpret_cast<float*>(smem);          // Hq * D floats (fits the K/V tiles)
    const int H = Hq * D;
    float am = 0.f;
    for (int v = threadIdx.x; v < H / 8; v += 128) {
      const int e = v * 8, h = e / D, c = e % D;
      const uint4 ou = __ldcg(reinterpret_cast<const uint4*>(out + (size_t)tok * H + e));
      const uint4 gu = *reinterpret_cast<const uint4*>(ga.gate + (size_t)tok * ga.ldg +
                                                       (size_t)h * ga.ghs + c);
      const __nv_bfloat162* oh = reinterpret_cast<const __nv_bfloat162*>(&ou);
      const __nv_bfloat162* gh = reinterpret_cast<const __nv_bfloat162*>(&gu);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 of = __bfloat1622float2(oh[j]), gf = __bfloat1622float2(gh[j]);
        const float y0 = bf16_round(of.x / (1.f + __expf(-gf.x)));
        const float y1 = bf16_round(of.y / (1.f + __expf(-gf.y)));
        buf[e + 2 * j] = y0;
        buf[e + 2 * j + 1] = y1;
        am = fmaxf(am, fmaxf(fabsf(y0), fabsf(y1)));
      }
    }
    am = warp_max(am);
    if (lane == 0) s_fin[warp][0] = am;
    __syncthreads();
    am = fmaxf(fmaxf(s_fin[0][0], s_fin[1][0]), fmaxf(s_fin[2][0], s_fin[3][0]));
    const float qs = fmaxf(am / 448.f, 1.f / (448.f * 512.f));
    const float inv = 1.f / qs;
    for (int v = threadIdx.x; v < H / 8; v += 128) {
      uint2 qq;
      uint16_t* q16 = reinterpret_cast<uint16_t*>(&qq);
#pragma unroll
      for (int j = 0; j < 4; ++j) q16[j] = f32x2_to_e4m3x2(buf[v * 8 + 2 * j] * inv, buf[v * 8 + 2 * j + 1] * inv);
      *reinterpret_cast<uint2*>(ga.q + (size_t)tok * ga.ldq + v * 8) = qq;
    }
    if (threadIdx.x == 0) ga.q_scale[tok] = qs;
  }
}

// merge split partials: one warp per (token, head)
template <int D>
__global__ void attn_merge_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                                  int num_splits, int T, int Hq, __nv_bfloat16* __restrict__ out) {
  pdl_wait();     // inputs come from the preceding kernel
  pdl_trigger();
  const int gw = blockIdx.x * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (gw >= T * Hq) return;
  float mmax = -INFINITY;
  for (int s = 0; s < num_splits; ++s) {
    const float m = part_ml[((size_t)s * T * Hq + gw) * 2];
    const float l = part_ml[((size_t)s * T * Hq + gw) * 2 + 1];
    if (l > 0.f) mmax = fmaxf(mmax, m);
  }
  constexpr int PER = D / 32;
  float acc[PER];
#pragma unroll
  for (int p = 0; p < PER; ++p) acc[p] = 0.f;
  float wsum = 0.f;
  for (int s = 0; s < num_splits; ++s) {
    const float m = part_ml[((size_t)s * T * Hq + gw) * 2];
    const float l = part_ml[((size_t)s * T * Hq + gw) * 2 + 1];
    if (!(l > 0.f)) continue;
    const float w = l * exp2f(m - mmax);
    wsum += w;
    const float* src = part_o + ((size_t)s * T * Hq + gw) * D;
#pragma unroll
    for (int p = 0; p < PER; ++p) acc[p] += w * src[lane * PER + p];
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
#pragma unroll
  for (int p = 0; p < PER; ++p) out[(size_t)gw * D + lane * PER + p] = __float2bfloat16_rn(acc[p] * inv);
}

}  // namespace attn

void qkv_prologue(torch::Tensor qkv, int64_t q_head_stride, int64_t k_off, int64_t v_off,
                  torch::Tensor positions, torch::Tensor qn_w, torch::Tensor kn_w,
                  torch::Tensor cos_sin, int64_t rot, int64_t Hq, int64_t Hkv, double eps,
                  torch::Tensor q_out, torch::Tensor k_cache, torch::Tensor v_cache,
                  torch::Tensor slot_mapping) {
  const int T = qkv.size(0);
  if (T == 0) return;
  const int D = q_out.size(2);
  const int block_size = k_cache.size(2);
  const int fmt = k_cache.scalar_type() == at::kFloat8_e4m3fn ? 1
                : k_cache.scalar_type() == at::kByte ? 2 : 0;
  TORCH_CHECK(positions.scalar_type() == at::kInt && slot_mapping.scalar_type() == at::kLong, "index dtypes");
  TORCH_CHECK(((rot / 2) % (D / 32)) == 0, "rotary dim / lanes");
  const at::cuda::CUDAGuard guard(qkv.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int warps = T * (Hq + Hkv);
  dim3 grid((warps + 7) / 8);
  auto run = [&](auto dtag) {
    constexpr int Dc = decltype(dtag)::value;
C10_CUDA_CHECK(launch_pdl((attn::qkv_prologue_kernel<Dc>), dim3(grid), dim3(256), 0, stream, 
        (const __nv_bfloat16*)qkv.data_ptr(), qkv.stride(0), q_head_stride, k_off, v_off,
        positions.data_ptr<int>(), (const __nv_bfloat16*)qn_w.data_ptr(),
        (const __nv_bfloat16*)kn_w.data_ptr(), cos_sin.data_ptr<float>(), rot, T, Hq, Hkv,
        (float)eps, (__nv_bfloat16*)q_out.data_ptr(), (uint8_t*)k_cache.data_ptr(),
        (uint8_t*)v_cache.data_ptr(), fmt, slot_mapping.data_ptr<int64_t>(), block_size));
  };
  if (D == 256) run(std::integral_constant<int, 256>{});
  else if (D == 128) run(std::integral_constant<int, 128>{});
  else if (D == 64) run(std::integral_constant<int, 64>{});
  else TORCH_CHECK(false, "qkv_prologue: head_dim 64/128/256");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// q [T, Hq, D] bf16; caches [blocks, Hkv, block_size(=64k), D]; tile_seq/tile_row0 [num_tiles];
// part_o [splits, T, Hq, D] fp32 and part_ml [splits, T, Hq, 2] (used when num_splits > 1).
// With gq defined (decode kernel, one token per tile): the o_proj producer runs in the same
// launch -- gate [T, *] bf16 (head h at column h * gate_head_stride), gate_cnt int32 [T] zero
// counters, gq e4m3 [T, Hq * D] and gq_scale [T] receive the gated, quantised rows.
void paged_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                     torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor qsl,
                     torch::Tensor tile_seq, torch::Tensor tile_row0, double scale, bool causal,
                     int64_t window, int64_t num_splits, torch::Tensor part_o,
                     torch::Tensor part_ml, torch::Tensor out, torch::Tensor counters,
                     bool decode, torch::Tensor gate, int64_t gate_head_stride,
                     torch::Tensor gate_cnt, torch::Tensor gq, torch::Tensor gq_scale) {
  const int T = q.size(0), Hq = q.size(1), D = q.size(2);
  const int Hkv = k_cache.size(1), block_size = k_cache.size(2);
  const int num_tiles = tile_seq.size(0);
  if (T == 0 || num_tiles == 0) return;
  TORCH_CHECK(block_size % attn::BC == 0 || attn::BC % block_size == 0,
              "KV page size must divide or be a multiple of 64");
  TORCH_CHECK(num_splits >= 1 && num_splits <= (decode ? 128 : 32),
              "num_splits must be in [1, 32] (decode kernel: [1, 128])");
  const int fmt = k_cache.scalar_type() == at::kFloat8_e4m3fn ? 1
                : k_cache.scalar_type() == at::kByte ? 2 : 0;
  const bool gated = gq.defined() && gq.numel();
  attn::AttnGateArgs ga{};
  if (gated) {
    TORCH_CHECK(decode, "paged_attention: the fused gate needs the decode kernel");
    TORCH_CHECK(out.is_contiguous() && (int64_t)Hq * D * 4 <= (16 + 2 * attn::BC) * D * 2,
                "paged_attention: fused gate row");
    TORCH_CHECK(gate.scalar_type() == at::kBFloat16 && gate.stride(1) == 1 && gate.stride(0) % 8 == 0 &&
                    gate_head_stride % 8 == 0 &&
                    (reinterpret_cast<uintptr_t>(gate.data_ptr()) % 16) == 0, "paged_attention: gate");
    TORCH_CHECK(gq.scalar_type() == at::kFloat8_e4m3fn && gq.stride(1) == 1 && gq.stride(0) % 8 == 0 &&
                    gq.size(1) >= Hq * D, "paged_attention: gq");
    TORCH_CHECK(gate_cnt.numel() >= T && gq_scale.numel() >= T, "paged_attention: gate counters");
    ga.gate = (const __nv_bfloat16*)gate.data_ptr();
    ga.ldg = (int)gate.stride(0);
    ga.ghs = (int)gate_head_stride;
    ga.tok_cnt = reinterpret_cast<unsigned*>(gate_cnt.data_ptr<int>());
    ga.q = (uint8_t*)gq.data_ptr();
    ga.ldq = (int)gq.stride(0);
    ga.q_scale = gq_scale.data_ptr<float>();
  }
  const at::cuda::CUDAGuard guard(q.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const float scale_log2 = (float)(scale * 1.4426950408889634);
  dim3 grid(num_tiles, Hkv, num_splits);
  auto run = [&](auto dtag, auto ftag) {
    constexpr int Dc = decltype(dtag)::value;
    constexpr int F8 = decltype(ftag)::value;
    // decode: tiles hold at most 16 query rows (the caller guarantees G * q_len <= 16)
    const int smem = ((decode ? 16 : attn::BR) + 2 * attn::BC) * Dc * 2;
    const __nv_bfloat16* qp = (const __nv_bfloat16*)q.data_ptr();
    const uint8_t* kp = (const uint8_t*)k_cache.data_ptr();
    const uint8_t* vp = (const uint8_t*)v_cache.data_ptr();
    float* po = num_splits > 1 ? part_o.data_ptr<float>() : nullptr;
    float* pm = num_splits > 1 ? part_ml.data_ptr<float>() : nullptr;
    unsigned* cn = num_splits > 1 ? reinterpret_cast<unsigned*>(counters.data_ptr()) : nullptr;
    if (decode) {
      auto kern = gated ? attn::paged_attn_decode_kernel<Dc, F8, true>
                        : attn::paged_attn_decode_kernel<Dc, F8, false>;
      static bool set[2] = {false, false};
      if (!set[gated]) {
        C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        set[gated] = true;
      }
      C10_CUDA_CHECK(launch_pdl(kern, dim3(grid), dim3(128), smem, stream, qp, kp, vp,
          block_tables.data_ptr<int>(), block_tables.stride(0), seq_lens.data_ptr<int>(),
          qsl.data_ptr<int>(), tile_seq.data_ptr<int>(), tile_row0.data_ptr<int>(), Hq, Hkv,
          block_size, scale_log2, causal ? 1 : 0, (int)window, (int)num_splits,
          (__nv_bfloat16*)out.data_ptr(), po, pm, T, cn, ga));
    } else {
      auto kern = attn::paged_attn_kernel<Dc, F8>;
      static bool set = false;
      if (!set) {
        C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        set = true;
      }
      C10_CUDA_CHECK(launch_pdl(kern, dim3(grid), dim3(128), smem, stream, qp, kp, vp,
          block_tables.data_ptr<int>(), block_tables.stride(0), seq_lens.data_ptr<int>(),
          qsl.data_ptr<int>(), tile_seq.data_ptr<int>(), tile_row0.data_ptr<int>(), Hq, Hkv,
          block_size, scale_log2, causal ? 1 : 0, (int)window, (int)num_splits,
          (__nv_bfloat16*)out.data_ptr(), po, pm, T, cn));
    }
  };
  auto by_fmt = [&](auto dtag) {
    if (fmt == 1) run(dtag, std::integral_constant<int, 1>{});
    else if (fmt == 2) run(dtag, std::integral_constant<int, 2>{});
    else run(dtag, std::integral_constant<int, 0>{});
  };
  if (D == 256) by_fmt(std::integral_constant<int, 256>{});
  else if (D == 128) by_fmt(std::integral_constant<int, 128>{});
  else if (D == 64) by_fmt(std::integral_constant<int, 64>{});
  else TORCH_CHECK(false, "paged_attention: head_dim 64/128/256");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace rad
