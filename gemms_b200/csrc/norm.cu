// norm.cu -- the steps either side of the MoE layer: RMSNorm fused with the
// per-1x128 FP8 activation quantisation before it.
//
// The reference's operator starts from already-quantised activations
// (flashinfer_baseline.py:5-16, hidden_states + hidden_states_scale); in the
// DeepSeek-V3 decoder the MoE input is the post-attention RMSNorm of the
// residual stream.  One pass here produces both inputs the layer needs: the
// bf16 normalised rows y (the router GEMM's input) and their e4m3 1x128
// quantisation with scales [H/128, T] (the experts' input, the layout of the
// reference's hidden_states_scale), so the layer does not quantise again.
//
// RMSNorm as DeepSeek-V3 defines it: v = mean(h^2) in fp32,
// y = weight * bf16(h * rsqrt(v + eps)) with the product rounded to bf16.
// The residual add after the layer is fused into the layer's output cast
// (to_bf16_kernel in permute.cu).
#include "common.cuh"

#include <algorithm>

namespace gemms {
namespace {

__device__ __forceinline__ uint32_t pack_e4m3x4(float v0, float v1, float v2, float v3, float scale) {
  const __nv_fp8x2_storage_t lo =
      __nv_cvt_float2_to_fp8x2(make_float2(__fdiv_rn(v0, scale), __fdiv_rn(v1, scale)), __NV_SATFINITE, __NV_E4M3);
  const __nv_fp8x2_storage_t hi =
      __nv_cvt_float2_to_fp8x2(make_float2(__fdiv_rn(v2, scale), __fdiv_rn(v3, scale)), __NV_SATFINITE, __NV_E4M3);
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

// One CTA (256 threads) per token row.  Pass 1: sum of squares (each thread
// over 16-column chunks, then a block reduction in a fixed order).  Pass 2
// (the row is re-read from L1/L2): normalise, round to bf16, multiply by the
// weight, round to bf16, and quantise each 128-column block (its 8 chunks sit
// in 8 consecutive lanes, which exchange their amax with three shuffles).
__global__ void __launch_bounds__(256) rmsnorm_quant_kernel(const __nv_bfloat16* __restrict__ h, const void* weight,
                                                            int weight_bf16, float eps, int T, int H,
                                                            __nv_bfloat16* __restrict__ y, uint8_t* __restrict__ xq,
                                                            float* __restrict__ xq_scale) {
  __shared__ float s_part[8];
  const int t = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int chunks = H / 16;
  const __nv_bfloat16* row = h + (size_t)t * H;

  float ss = 0.f;
  for (int c = tid; c < chunks; c += blockDim.x) {
    const uint4* src = reinterpret_cast<const uint4*>(row + 16 * (size_t)c);
    const uint4 r0 = src[0], r1 = src[1];
    const uint32_t u[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[k]));
      ss = fmaf(v.x, v.x, ss);
      ss = fmaf(v.y, v.y, ss);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if (lane == 0) s_part[warp] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += s_part[w];
  const float r = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)H), eps)));

  // Pass 2: whole warps iterate together (the amax shuffles need all lanes).
  for (int c0 = 0; c0 < chunks; c0 += blockDim.x) {
    const int c = c0 + tid;
    const bool live = c < chunks;
    const int cc = live ? c : chunks - 1;
    const uint4* src = reinterpret_cast<const uint4*>(row + 16 * (size_t)cc);
    const uint4 r0 = src[0], r1 = src[1];
    const uint32_t u[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
    float v[16];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float2 hv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[k]));
      const int col = 16 * cc + 2 * k;
      float w0, w1;
      if (weight_bf16) {
        const __nv_bfloat162 wb = reinterpret_cast<const __nv_bfloat162*>(weight)[col / 2];
        w0 = __low2float(wb);
        w1 = __high2float(wb);
      } else {
        const float2 wf = reinterpret_cast<const float2*>(weight)[col / 2];
        w0 = wf.x;
        w1 = wf.y;
      }
      // bf16(h * r), then times the weight, rounded to bf16
      const float n0 = __bfloat162float(__float2bfloat16_rn(__fmul_rn(hv.x, r)));
      const float n1 = __bfloat162float(__float2bfloat16_rn(__fmul_rn(hv.y, r)));
      v[2 * k] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(w0, n0)));
      v[2 * k + 1] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(w1, n1)));
    }
    if (live && y) {
      uint4 o0, o1;
      uint32_t* po = &o0.x;
      uint32_t* pp = &o1.x;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const __nv_bfloat162 a = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
        const __nv_bfloat162 b = __floats2bfloat162_rn(v[8 + 2 * k], v[8 + 2 * k + 1]);
        po[k] = *reinterpret_cast<const uint32_t*>(&a);
        pp[k] = *reinterpret_cast<const uint32_t*>(&b);
      }
      uint4* dst = reinterpret_cast<uint4*>(y + (size_t)t * H + 16 * (size_t)c);
      dst[0] = o0;
      dst[1] = o1;
    }
    if (xq) {
      float amax = 0.f;
#pragma unroll
      for (int k = 0; k < 16; ++k) amax = fmaxf(amax, fabsf(v[k]));
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
      const float scale = amax > 0.f ? __fdiv_rn(amax, kFp8Max) : 1.0f;
      if (live) {
        uint4 q;
        q.x = pack_e4m3x4(v[0], v[1], v[2], v[3], scale);
        q.y = pack_e4m3x4(v[4], v[5], v[6], v[7], scale);
        q.z = pack_e4m3x4(v[8], v[9], v[10], v[11], scale);
        q.w = pack_e4m3x4(v[12], v[13], v[14], v[15], scale);
        *reinterpret_cast<uint4*>(xq + (size_t)t * H + 16 * (size_t)c) = q;
        if ((c & 7) == 0) xq_scale[(size_t)(c >> 3) * T + t] = scale;
      }
    }
  }
}

}  // namespace
}  // namespace gemms

extern "C" int gemms_rmsnorm_quant(const void* h_bf16, const void* weight, int32_t weight_bf16, float eps, int32_t T,
                                   int32_t H, void* y_bf16, void* xq, float* xq_scale, gemms_stream_t stream) {
  using namespace gemms;
  if (T < 0 || H <= 0 || H % kBlock || !(eps >= 0.f)) return GEMMS_ERR_SHAPE;
  if (T == 0) return GEMMS_OK;
  if (!h_bf16 || !weight || (!y_bf16 && !xq) || (xq && !xq_scale)) return GEMMS_ERR_ARG;
  if (!aligned16(h_bf16) || (y_bf16 && !aligned16(y_bf16)) || (xq && !aligned16(xq)) ||
      (reinterpret_cast<uintptr_t>(weight) & 7u))
    return GEMMS_ERR_ALIGN;
  rmsnorm_quant_kernel<<<T, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(h_bf16), weight, weight_bf16, eps, T, H, static_cast<__nv_bfloat16*>(y_bf16),
      static_cast<uint8_t*>(xq), xq_scale);
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}
