// Quantised token-embedding lookup: the table is stored as int8 with one fp32 scale per row, or
// as 4-bit codes (two per byte, low nibble = even column, value = code - 8) with one bf16 scale
// per 128 columns; the gather dequantises straight into the bf16 rows of the step.
//
// Reference behaviour: sly/mxfp4/radiance_embed_int8.py:47-114 (per-row int8 or g128 int4
// embed_tokens, quantised at load, dequantised on lookup).  Here the lookup is one kernel: a CTA
// per token streams its row with 16-byte loads and writes bf16 (no index_select + elementwise
// chain).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace rad {
namespace emb {

// int8: 16 codes per thread step
__global__ void __launch_bounds__(128) gather_int8_kernel(
    const int8_t* __restrict__ codes, const float* __restrict__ scales,
    const int64_t* __restrict__ ids, int V, int H, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  int64_t id = ids[t];
  id = id < 0 ? 0 : (id >= V ? V - 1 : id);          // out-of-range ids clamp (no fault)
  const float s = scales[id];
  const int8_t* row = codes + (size_t)id * H;
  for (int v = threadIdx.x; v < H / 16; v += blockDim.x) {
    const int4 u = *reinterpret_cast<const int4*>(row + v * 16);
    const int8_t* b = reinterpret_cast<const int8_t*>(&u);
    uint4 o[2];
    __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(o);
#pragma unroll
    for (int i = 0; i < 8; ++i) oh[i] = __floats2bfloat162_rn((float)b[2 * i] * s, (float)b[2 * i + 1] * s);
    uint4* dst = reinterpret_cast<uint4*>(out + (size_t)t * H + v * 16);
    dst[0] = o[0];
    dst[1] = o[1];
  }
}

// int4 g128: 16 codes (8 bytes) per thread step, all inside one 128-column group
__global__ void __launch_bounds__(128) gather_int4_kernel(
    const uint8_t* __restrict__ codes, const __nv_bfloat16* __restrict__ scales,
    const int64_t* __restrict__ ids, int V, int H, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  int64_t id = ids[t];
  id = id < 0 ? 0 : (id >= V ? V - 1 : id);
  const uint8_t* row = codes + (size_t)id * (H / 2);
  const __nv_bfloat16* srow = scales + (size_t)id * (H / 128);
  for (int v = threadIdx.x; v < H / 16; v += blockDim.x) {
    const uint2 u = *reinterpret_cast<const uint2*>(row + v * 8);
    const uint8_t* b = reinterpret_cast<const uint8_t*>(&u);
    const float s = __bfloat162float(srow[(v * 16) / 128]);
    uint4 o[2];
    __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(o);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      oh[i] = __floats2bfloat162_rn((float)((int)(b[i] & 0xF) - 8) * s, (float)((int)(b[i] >> 4) - 8) * s);
    uint4* dst = reinterpret_cast<uint4*>(out + (size_t)t * H + v * 16);
    dst[0] = o[0];
    dst[1] = o[1];
  }
}

}  // namespace emb

// ids [T] int64 -> out [T, H] bf16.  bits 8: codes int8 [V, H], scales fp32 [V];
// bits 4: codes uint8 [V, H / 2], scales bf16 [V, H / 128].
void embed_gather(torch::Tensor codes, torch::Tensor scales, torch::Tensor ids, int64_t bits,
                  torch::Tensor out) {
  const int T = ids.size(0);
  const int V = codes.size(0);
  const int H = out.size(1);
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.size(0) >= T,
              "embed_gather: out");
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous(), "embed_gather: int64 ids");
  TORCH_CHECK(H % 128 == 0, "embed_gather: hidden size a multiple of 128");
  TORCH_CHECK(codes.is_contiguous() && scales.is_contiguous(), "embed_gather: contiguous table");
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(out.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  if (bits == 8) {
    TORCH_CHECK(codes.scalar_type() == at::kChar && codes.size(1) == H &&
                    scales.scalar_type() == at::kFloat && scales.numel() >= V, "embed_gather: int8 table");
    C10_CUDA_CHECK(launch_pdl(emb::gather_int8_kernel, dim3(T), dim3(128), 0, stream,
                              (const int8_t*)codes.data_ptr(), scales.data_ptr<float>(),
                              ids.data_ptr<int64_t>(), V, H, (__nv_bfloat16*)out.data_ptr()));
  } else {
    TORCH_CHECK(bits == 4 && codes.scalar_type() == at::kByte && codes.size(1) == H / 2 &&
                    scales.scalar_type() == at::kBFloat16 && scales.size(1) == H / 128,
                "embed_gather: int4 g128 table");
    C10_CUDA_CHECK(launch_pdl(emb::gather_int4_kernel, dim3(T), dim3(128), 0, stream,
                              (const uint8_t*)codes.data_ptr(),
                              (const __nv_bfloat16*)scales.data_ptr(), ids.data_ptr<int64_t>(), V,
                              H, (__nv_bfloat16*)out.data_ptr()));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace rad
