// permute.cu -- token -> expert-grouped row gather with fused per-1x128 FP8
// activation quantisation, and the fp32 -> bf16 output cast.
//
// Reference: the oracle gathers rows per expert with index_select
// (flashinfer_baseline.py:141-149) after dequantising [T,H] e4m3 activations
// with a transposed [H/128, T] scale (:68-79).  The build stores the grouped
// operand with the same transposed scale layout, [H/128, rows], so a GEMM
// epilogue warp reads the scales of 32 consecutive rows as one coalesced load.
#include "common.cuh"

#include <algorithm>

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

// Block (t, y) of 8 warps handles token t; warp w takes the 128-column blocks
// y*8 + w, y*8 + w + 8*gridDim.y, ...
// Each lane owns 4 consecutive columns of a block, so a warp writes one
// 128-byte line per destination row.
__global__ void __launch_bounds__(256) permute_kernel(PermuteArgs a) {
  constexpr int kMaxDst = 17;  // top_k <= 16 + the shared expert
  __shared__ int s_dst[kMaxDst];
  __shared__ int s_nd;
  const int t = blockIdx.x;
  if (a.T_dev && t >= *a.T_dev) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (warp == 0) {  // the token's grouped rows, compacted in slot order
    const int r = lane < a.top_k ? a.pair_row[(size_t)t * a.top_k + lane] : -1;
    const unsigned b = __ballot_sync(0xffffffffu, r >= 0);
    if (r >= 0) s_dst[__popc(b & ((1u << lane) - 1u))] = r;
    int nd = __popc(b);
    if (lane == 0) {
      if (a.shared_row0) s_dst[nd++] = *a.shared_row0 + t;
      s_nd = nd;
    }
  }
  __syncthreads();
  const int nd = s_nd;
  const int* dst = s_dst;
  if (nd == 0) return;
  const int KB = a.H / kBlock;
  for (int kb = blockIdx.y * 8 + warp; kb < KB; kb += 8 * gridDim.y) {
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

// Token-major per-1x128 quantisation: x bf16 [T, H] -> xq e4m3 [T, H] and
// xq_scale fp32 [H/128, T] (the reference's transposed hidden_states_scale
// layout, flashinfer_baseline.py:59,72).  A thread owns 16 consecutive
// columns (two 16-byte loads, one 16-byte store); the 8 threads of a
// 128-column block exchange their amax with three shuffles.
__global__ void __launch_bounds__(256) quantize_kernel(const __nv_bfloat16* __restrict__ x, int T, int H,
                                                       uint8_t* __restrict__ xq, float* __restrict__ xq_scale) {
  const int per_row = H / 16;
  const size_t total = (size_t)T * per_row;
  // Whole warps iterate together (the shuffles below need all 32 lanes).
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i0 = (size_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31u); i0 < total; i0 += stride) {
    const size_t i = i0 + (threadIdx.x & 31);
    const bool live = i < total;
    const size_t ii = live ? i : total - 1;
    const int t = static_cast<int>(ii / per_row);
    const int c16 = static_cast<int>(ii - (size_t)t * per_row);
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)t * H + 16 * (size_t)c16);
    const uint4 r0 = src[0], r1 = src[1];
    float v[16];
    const uint32_t w[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&w[k]);
      v[2 * k] = __low2float(b);
      v[2 * k + 1] = __high2float(b);
    }
    float amax = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) amax = fmaxf(amax, fabsf(v[k]));
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const float scale = amax > 0.f ? __fdiv_rn(amax, kFp8Max) : 1.0f;
    uint4 q;
    q.x = quant4(v[0], v[1], v[2], v[3], scale);
    q.y = quant4(v[4], v[5], v[6], v[7], scale);
    q.z = quant4(v[8], v[9], v[10], v[11], scale);
    q.w = quant4(v[12], v[13], v[14], v[15], scale);
    if (live) {
      *reinterpret_cast<uint4*>(xq + (size_t)t * H + 16 * (size_t)c16) = q;
      if ((c16 & 7) == 0) xq_scale[(size_t)(c16 >> 3) * T + t] = scale;
    }
  }
}

__global__ void to_bf16_kernel(const float4* __restrict__ in, uint2* __restrict__ out, size_t n4,
                               const uint2* __restrict__ residual) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    float4 v = in[i];
    if (residual) {  // the decoder's residual add, fused: one rounding of (residual + layer)
      const uint2 r = residual[i];
      const float2 r0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.x));
      const float2 r1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.y));
      v.x += r0.x;
      v.y += r0.y;
      v.z += r1.x;
      v.w += r1.y;
    }
    __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y);
    __nv_bfloat162 b = __floats2bfloat162_rn(v.z, v.w);
    uint2 o;
    o.x = *reinterpret_cast<uint32_t*>(&a);
    o.y = *reinterpret_cast<uint32_t*>(&b);
    out[i] = o;
  }
}

// Block per token: the token's slot rows (its top-k grouped rows in slot
// order, then the shared expert's) are summed in that fixed order, so the
// result does not depend on which CTA finished first.
__global__ void __launch_bounds__(256, 4) combine_slots_kernel(const float* __restrict__ pair_out,
                                                               const int32_t* __restrict__ pair_row, int T, int K,
                                                               int H, const int32_t* __restrict__ shared_row0,
                                                               const uint2* __restrict__ residual,
                                                               uint2* __restrict__ out_bf16,
                                                               float4* __restrict__ out_f32,
                                                               const int32_t* __restrict__ T_dev) {
  __shared__ int s_rows[17];
  __shared__ int s_n;
  const int t = blockIdx.x;
  if (T_dev && t >= *T_dev) return;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x < 32) {
    const int r = lane < K ? pair_row[(size_t)t * K + lane] : -1;
    const unsigned b = __ballot_sync(0xffffffffu, r >= 0);
    if (r >= 0) s_rows[__popc(b & ((1u << lane) - 1u))] = r;
    if (lane == 0) {
      int n = __popc(b);
      if (shared_row0) s_rows[n++] = *shared_row0 + t;
      s_n = n;
    }
  }
  __syncthreads();
  const int n = s_n;
  const int H4 = H / 4;
  for (int c = threadIdx.x; c < H4; c += blockDim.x) {
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = 0; i < n; ++i) {
      const float4 x = reinterpret_cast<const float4*>(pair_out + (size_t)s_rows[i] * H)[c];
      v.x += x.x;
      v.y += x.y;
      v.z += x.z;
      v.w += x.w;
    }
    const size_t o = (size_t)t * H4 + c;
    if (out_f32) {
      out_f32[o] = v;
      continue;
    }
    if (residual) {
      const uint2 rr = residual[o];
      const float2 r0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&rr.x));
      const float2 r1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&rr.y));
      v.x += r0.x;
      v.y += r0.y;
      v.z += r1.x;
      v.w += r1.y;
    }
    __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y);
    __nv_bfloat162 b = __floats2bfloat162_rn(v.z, v.w);
    uint2 w;
    w.x = *reinterpret_cast<uint32_t*>(&a);
    w.y = *reinterpret_cast<uint32_t*>(&b);
    out_bf16[o] = w;
  }
}
}  // namespace

int launch_permute(const PermuteArgs& a, cudaStream_t s) {
  if (a.T <= 0) return GEMMS_OK;
  if (a.top_k > 16) return GEMMS_ERR_SHAPE;
  // Few tokens (decode): split each token's 128-column blocks over several
  // blocks, one column block per warp, so that the copy is not one block's
  // serial loop.
  const int col_blocks = a.T < 4 * num_sms() ? cdiv(a.H / kBlock, 8) : 1;
  permute_kernel<<<dim3(a.T, col_blocks), 256, 0, s>>>(a);
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}

int launch_quantize(const __nv_bfloat16* x, int T, int H, uint8_t* xq, float* xq_scale, cudaStream_t s) {
  if (T <= 0) return GEMMS_OK;
  if (H % kBlock) return GEMMS_ERR_SHAPE;
  if (!aligned16(x) || !aligned16(xq)) return GEMMS_ERR_ALIGN;
  const size_t total = (size_t)T * (H / 16);
  const int blocks = static_cast<int>(std::min<size_t>((total + 255) / 256, (size_t)num_sms() * 16));
  quantize_kernel<<<blocks, 256, 0, s>>>(x, T, H, xq, xq_scale);
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}

int launch_to_bf16(const float* in, __nv_bfloat16* out, size_t n, const __nv_bfloat16* residual, cudaStream_t s) {
  if (n == 0) return GEMMS_OK;
  if (n % 4) return GEMMS_ERR_SHAPE;
  if (residual && (reinterpret_cast<uintptr_t>(residual) & 7u)) return GEMMS_ERR_ALIGN;
  const size_t n4 = n / 4;
  const int blocks = static_cast<int>(std::min<size_t>((n4 + 255) / 256, (size_t)num_sms() * 8));
  to_bf16_kernel<<<blocks, 256, 0, s>>>(reinterpret_cast<const float4*>(in), reinterpret_cast<uint2*>(out), n4,
                                        reinterpret_cast<const uint2*>(residual));
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}

int launch_combine_slots(const float* pair_out, const int32_t* pair_row, int T, int K, int H,
                         const int32_t* shared_row0, const __nv_bfloat16* residual, __nv_bfloat16* out_bf16,
                         float* out_f32, const int32_t* T_dev, cudaStream_t s) {
  if (T <= 0) return GEMMS_OK;
  if (H % 4 || K < 1 || K > 16 || (!out_bf16 && !out_f32)) return GEMMS_ERR_SHAPE;
  if ((residual && (reinterpret_cast<uintptr_t>(residual) & 7u)) || !aligned16(pair_out) ||
      (out_f32 && !aligned16(out_f32)) || (out_bf16 && (reinterpret_cast<uintptr_t>(out_bf16) & 7u)))
    return GEMMS_ERR_ALIGN;
  combine_slots_kernel<<<T, 256, 0, s>>>(pair_out, pair_row, T, K, H, shared_row0,
                                         reinterpret_cast<const uint2*>(residual), reinterpret_cast<uint2*>(out_bf16),
                                         reinterpret_cast<float4*>(out_f32), T_dev);
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}

}  // namespace gemms

extern "C" int gemms_quantize_1x128(const void* x_bf16, int32_t T, int32_t H, void* xq, float* xq_scale,
                                    gemms_stream_t stream) {
  if (T < 0 || H <= 0 || H % gemms::kBlock) return GEMMS_ERR_SHAPE;
  if (T == 0) return GEMMS_OK;
  if (!x_bf16 || !xq || !xq_scale) return GEMMS_ERR_ARG;
  return gemms::launch_quantize(static_cast<const __nv_bfloat16*>(x_bf16), T, H, static_cast<uint8_t*>(xq), xq_scale,
                                reinterpret_cast<cudaStream_t>(stream));
}
