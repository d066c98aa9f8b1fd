// permute.cu -- token -> expert-grouped row gather with fused per-1x128 FP8
// activation quantisation, and the fp32 -> bf16 output cast.
//
// Reference: the oracle gathers rows per expert with index_select
// (flashinfer_baseline.py:141-149) after dequantising [T,H] e4m3 activations
// with a transposed [H/128, T] scale (:68-79).  The build stores the grouped
// operand with the same transposed scale layout, [H/128, rows], so a GEMM
// epilogue warp reads the scales of 32 consecutive rows as one coalesced load.
#include "common.cuh"

namespace gemms {
namespace {

__device__ __forceinline__ uint32_t quant4(float v0, float v1, float v2, float v3, float scale) {
  // e4m3 round-to-nearest-even with saturation; same bytes as torch's
  // (x / scale).to(float8_e4m3fn) for |x / scale| <= 448.
  const __nv_fp8x2_storage_t lo =
      __nv_cvt_float2_to_fp8x2(make_float2(__fdiv_rn(v0, scale), __fdiv_rn(v1, scale)), __NV_SATFINITE, __NV_E4M3);
  const __nv_fp8x2_storage_t hi =
      __nv_cvt_float2_to_fp8x2(make_float2(__fdiv_rn(v2, scale), __fdiv_rn(v3, scale)), __NV_SATFINITE, __NV_E4M3);
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

// One block of 8 warps per token; warp w handles 128-column blocks w, w+8, ...
// Each lane owns 4 consecutive columns of a block, so a warp writes one
// 128-byte line per destination row.
__global__ void __launch_bounds__(256) permute_kernel(PermuteArgs a) {
  const int t = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int kMaxDst = 17;
  int dst[kMaxDst];
  int nd = 0;
  for (int j = 0; j < a.top_k; ++j) {
    const int r = a.pair_row[(size_t)t * a.top_k + j];
    if (r >= 0) dst[nd++] = r;
  }
  if (a.shared_row0) dst[nd++] = *a.shared_row0 + t;
  if (nd == 0) return;
  const int KB = a.H / kBlock;
  for (int kb = warp; kb < KB; kb += 8) {
    const size_t src = (size_t)t * a.H + (size_t)kb * kBlock + lane * 4;
    uint32_t packed;
    float scale;
    if (a.mode == GEMMS_INPUT_BF16) {
      const uint2 raw = *reinterpret_cast<const uint2*>(a.x_bf16 + src);
      const __nv_bfloat162 p0 = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
      const __nv_bfloat162 p1 = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
      const float v0 = __low2float(p0), v1 = __high2float(p0), v2 = __low2float(p1), v3 = __high2float(p1);
      float amax = fmaxf(fmaxf(fabsf(v0), fabsf(v1)), fmaxf(fabsf(v2), fabsf(v3)));
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
      scale = amax > 0.f ? __fdiv_rn(amax, kFp8Max) : 1.0f;
      packed = quant4(v0, v1, v2, v3, scale);
    } else {
      const long long rs = a.x_row_stride > 0 ? a.x_row_stride : a.H;
      const long long skb = a.scale_kb_stride > 0 ? a.scale_kb_stride : a.T;
      const long long st = a.scale_t_stride > 0 ? a.scale_t_stride : 1;
      packed = *reinterpret_cast<const uint32_t*>(a.x_fp8 + (size_t)t * rs + (size_t)kb * kBlock + lane * 4);
      scale = a.x_scale[kb * skb + t * st];
    }
    for (int d = 0; d < nd; ++d) {
      const int r = dst[d];
      *reinterpret_cast<uint32_t*>(a.rows_fp8 + (size_t)r * a.H + (size_t)kb * kBlock + lane * 4) = packed;
      if (lane == 0) a.rows_scale[(size_t)kb * a.scale_ld + r] = scale;
    }
  }
}

__global__ void to_bf16_kernel(const float4* __restrict__ in, uint2* __restrict__ out, size_t n4) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    const float4 v = in[i];
    __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y);
    __nv_bfloat162 b = __floats2bfloat162_rn(v.z, v.w);
    uint2 o;
    o.x = *reinterpret_cast<uint32_t*>(&a);
    o.y = *reinterpret_cast<uint32_t*>(&b);
    out[i] = o;
  }
}

}  // namespace

int launch_permute(const PermuteArgs& a, cudaStream_t s) {
  if (a.T <= 0) return GEMMS_OK;
  if (a.top_k > 16) return GEMMS_ERR_SHAPE;
  permute_kernel<<<a.T, 256, 0, s>>>(a);
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}

int launch_to_bf16(const float* in, __nv_bfloat16* out, size_t n, cudaStream_t s) {
  if (n == 0) return GEMMS_OK;
  if (n % 4) return GEMMS_ERR_SHAPE;
  const size_t n4 = n / 4;
  const int blocks = static_cast<int>(std::min<size_t>((n4 + 255) / 256, (size_t)num_sms() * 8));
  to_bf16_kernel<<<blocks, 256, 0, s>>>(reinterpret_cast<const float4*>(in), reinterpret_cast<uint2*>(out), n4);
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}

}  // namespace gemms
