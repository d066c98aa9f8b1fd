// decode.cu -- the two expert GEMMs for decode-sized batches (T <= 2) on the
// CUDA cores.
//
// With at most 2 rows per expert the tensor-core GEMMs (grouped_gemm.cu) run
// each M tile as one long chain of 128-deep K blocks per CTA, MMA -> TMEM ->
// promotion -> MMA, and at T=1 that chain, not HBM, sets their time (GEMM1:
// one 56-block chain per CTA).  Here the work is a weight stream: every weight
// byte is read once, converted from e4m3 and multiplied into <= 2 activation
// rows held in shared memory, with many 16-byte loads in flight per SM, so the
// time is the HBM time of the weights of the experts hit.
//
// Same operands and block-scale semantics as the tensor path (the reference's
// dequantise-then-matmul, flashinfer_baseline.py:68-93, 154-169): per
// 128-wide K block, sum(a_q * w_q) * a_scale[row, kb] * w_scale[n/128, kb],
// accumulated in fp32.  GEMM1 applies SwiGLU (silu on the second half,
// :157-160) and keeps the intermediate in fp32 (the reference's own precision;
// the tensor path re-quantises it to two e4m3 planes for its FP8 GEMM2).
// GEMM2 multiplies by the routing weight and adds into the token's fp32
// output row (or stores the row for the deterministic combine).
//
// Work: the M-tile list of plan_kernel (one tile per hit expert, since rows
// <= 2 < 128); a unit is (tile, a chunk of output rows); each CTA takes a
// contiguous range of units, so it re-stages the activation rows only when the
// tile changes.  Shared memory holds the activation rows as fp32 in a
// [row][element-in-chunk][chunk] layout: lane c of a warp reads chunk c, so a
// warp's shared loads hit 32 consecutive words (no bank conflicts).
#include "common.cuh"
#include "sm100.cuh"

#include <algorithm>
#include <atomic>

namespace gemms {
namespace {

constexpr int kDecThreads = 512;   // 16 warps
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kChunk = 16;         // weights per 16-byte load
constexpr int kRowsPerWarp = 4;    // GEMM1: 2 gate/up pairs; GEMM2: 4 output rows

__device__ __forceinline__ void e4m3x16_to_f(const uint4& w, float* f) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(
          static_cast<__nv_fp8x2_storage_t>((u[q] >> (16 * h)) & 0xffffu), __NV_E4M3);
      const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&hr));
      f[4 * q + 2 * h] = v.x;
      f[4 * q + 2 * h + 1] = v.y;
    }
  }
}

// 16-byte asynchronous copy global -> shared (L2 only): the weight stream is
// staged through a per-warp ring in shared memory, so the chunks in flight
// hold no registers.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t sa = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Ring stages per lane (chunks of the four weight rows in flight); fewer when
// four activation rows take most of the shared memory.
template <int MR>
constexpr int ring_stages() { return MR >= 4 ? 2 : 4; }
constexpr size_t ring_bytes(int stages) { return (size_t)kDecWarps * stages * kRowsPerWarp * 32 * 16; }

// (a0, a1) += (w0, w1) * (x0, x1): one packed fp32x2 FMA for two weights.
__device__ __forceinline__ void ffma2_vv(float& a0, float& a1, float w0, float w1, float x0, float x1) {
  asm("{\n\t.reg .b64 acc, wv, xv;\n\t"
      "mov.b64 acc, {%0, %1};\n\t"
      "mov.b64 wv, {%2, %3};\n\t"
      "mov.b64 xv, {%4, %5};\n\t"
      "fma.rn.f32x2 acc, wv, xv, acc;\n\t"
      "mov.b64 {%0, %1}, acc;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(w0), "f"(w1), "f"(x0), "f"(x1));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// Contiguous unit range of this CTA.
__device__ __forceinline__ void unit_range(int total, int& u0, int& u1) {
  const int per = (total + (int)gridDim.x - 1) / (int)gridDim.x;
  u0 = min(total, (int)blockIdx.x * per);
  u1 = min(total, u0 + per);
}

// GEMM1 + SwiGLU.  Unit = (tile, 32 intermediate columns j); warp w takes
// columns j0 + 2w and j0 + 2w + 1 (their gate rows j and up rows j + I).
// A 128-column block of one activation row, quantised per 1x128 exactly as
// permute_kernel does it: scale = amax / 448 (IEEE division), values
// v / scale (IEEE) rounded to e4m3 with saturation.  The 8 threads of a block
// (consecutive lanes) each hold 16 values and exchange their amax.
__device__ __forceinline__ float quantise16(float* f, bool valid) {
  float amax = 0.f;
#pragma unroll
  for (int e = 0; e < kChunk; ++e) amax = fmaxf(amax, fabsf(f[e]));
#pragma unroll
  for (int off = 1; off < 8; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  const float scale = amax > 0.f ? __fdiv_rn(amax, kFp8Max) : 1.0f;
#pragma unroll
  for (int e = 0; e < kChunk; e += 2) {
    const __nv_fp8x2_storage_t q = __nv_cvt_float2_to_fp8x2(
        make_float2(__fdiv_rn(f[e], scale), __fdiv_rn(f[e + 1], scale)), __NV_SATFINITE, __NV_E4M3);
    const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(q, __NV_E4M3);
    const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&hr));
    f[e] = valid ? d.x : 0.f;
    f[e + 1] = valid ? d.y : 0.f;
  }
  return valid ? scale : 0.f;
}

template <int MR>
__global__ void __launch_bounds__(kDecThreads, 1) decode_gemm1_kernel(Gemm1Args a, float* __restrict__ inter,
                                                                      DecodeSrc src) {
  extern __shared__ float smem[];
  const int H = a.H, I = a.I, KB = H / kBlock, NC = H / kChunk;
  float* sA = smem;                        // [MR][16][NC]
  float* sS = smem + (size_t)MR * H;       // [MR][KB] activation scales
  constexpr int S = ring_stages<MR>();
  uint4* ring = reinterpret_cast<uint4*>(smem + (((size_t)MR * (H + KB) + 3) & ~(size_t)3)) +
                (size_t)(threadIdx.x >> 5) * S * kRowsPerWarp * 32;  // this warp's [S][4][32] chunks
  const int num_tiles = min(*a.g.num_tiles, a.g.max_tiles);
  const int per_tile = I / (2 * kDecWarps);
  int u0, u1;
  unit_range(num_tiles * per_tile, u0, u1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int staged = -1;
  for (int u = u0; u < u1; ++u) {
    const int tile = u / per_tile, jc = u - tile * per_tile;
    const int g = a.g.tile_group[tile], row0 = a.g.tile_row0[tile], rows = min(a.g.tile_rows[tile], MR);
    if (tile != staged) {
      __syncthreads();  // previous tile's rows no longer read
      if (src.row_token) {
        // rows straight from the layer's input (token row_token[r]): no
        // permuted copy; whole warps iterate together for the amax exchange
        for (int i0 = 0; i0 < MR * NC; i0 += blockDim.x) {
          const int i = i0 + threadIdx.x;
          const int r = min(i / NC, MR - 1), c = i - (i / NC) * NC;
          const bool valid = i < MR * NC && r < rows;
          const int tok = valid ? src.row_token[row0 + r] : 0;
          float f[kChunk];
          float scale = 0.f;
          if (src.x_bf16) {
            const uint4* p = reinterpret_cast<const uint4*>(src.x_bf16 + (size_t)tok * H + (size_t)c * kChunk);
            const uint4 w0 = valid ? p[0] : make_uint4(0, 0, 0, 0), w1 = valid ? p[1] : make_uint4(0, 0, 0, 0);
            const uint32_t u[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int k2 = 0; k2 < 8; ++k2) {
              const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[k2]));
              f[2 * k2] = v.x;
              f[2 * k2 + 1] = v.y;
            }
            scale = quantise16(f, valid);
          } else {
            if (valid) {
              e4m3x16_to_f(*reinterpret_cast<const uint4*>(src.x_fp8 + (size_t)tok * H + (size_t)c * kChunk), f);
              scale = src.x_scale[(size_t)(c / (kBlock / kChunk)) * src.T + tok];
            } else {
#pragma unroll
              for (int e = 0; e < kChunk; ++e) f[e] = 0.f;
            }
          }
          if (i < MR * NC) {
#pragma unroll
            for (int e = 0; e < kChunk; ++e) sA[((size_t)r * kChunk + e) * NC + c] = f[e];
            if ((c & (kBlock / kChunk - 1)) == 0) sS[r * KB + c / (kBlock / kChunk)] = scale;
          }
        }
      } else {
        for (int i = threadIdx.x; i < MR * NC; i += blockDim.x) {
          const int r = i / NC, c = i - r * NC;
          float f[kChunk];
          if (r < rows) {
            e4m3x16_to_f(*reinterpret_cast<const uint4*>(a.a + (size_t)(row0 + r) * H + (size_t)c * kChunk), f);
          } else {
#pragma unroll
            for (int e = 0; e < kChunk; ++e) f[e] = 0.f;
          }
#pragma unroll
          for (int e = 0; e < kChunk; ++e) sA[((size_t)r * kChunk + e) * NC + c] = f[e];
        }
        for (int i = threadIdx.x; i < MR * KB; i += blockDim.x) {
          const int r = i / KB, kb = i - r * KB;
          sS[i] = r < rows ? a.a_scale[(size_t)kb * a.a_scale_ld + row0 + r] : 0.f;
        }
      }
      __syncthreads();
      staged = tile;
    }
    const bool sh = g == a.g.shared_group;
    const uint8_t* W = sh ? a.sw13 : a.w13 + (size_t)g * 2 * I * H;
    const float* WS = sh ? a.sw13_scale : a.w13_scale + (size_t)g * (2 * I / kBlock) * KB;
    const int j0 = jc * 2 * kDecWarps + 2 * warp;
    // weight rows: gate j0, gate j0+1, up j0, up j0+1
    const uint8_t* wrow[kRowsPerWarp] = {W + (size_t)j0 * H, W + (size_t)(j0 + 1) * H, W + (size_t)(I + j0) * H,
                                         W + (size_t)(I + j0 + 1) * H};
    const float* wsc[kRowsPerWarp] = {WS + (size_t)(j0 / kBlock) * KB, WS + (size_t)((j0 + 1) / kBlock) * KB,
                                      WS + (size_t)((I + j0) / kBlock) * KB,
                                      WS + (size_t)((I + j0 + 1) / kBlock) * KB};
    float acc[kRowsPerWarp][MR];
#pragma unroll
    for (int q = 0; q < kRowsPerWarp; ++q)
#pragma unroll
      for (int r = 0; r < MR; ++r) acc[q][r] = 0.f;
    // S - 1 chunks of the four rows in flight per lane through the ring
    const int n_it = (NC - lane + 31) / 32;  // chunks c = lane + 32 * it
#pragma unroll
    for (int st = 0; st < S - 1; ++st) {
      if (st < n_it) {
#pragma unroll
        for (int q = 0; q < kRowsPerWarp; ++q)
          cp_async16(ring + (st * kRowsPerWarp + q) * 32 + lane, wrow[q] + (size_t)(lane + 32 * st) * kChunk);
      }
      cp_async_commit();
    }
    for (int it = 0; it < n_it; ++it) {
      const int nx = it + S - 1;
      if (nx < n_it) {
#pragma unroll
        for (int q = 0; q < kRowsPerWarp; ++q)
          cp_async16(ring + ((nx % S) * kRowsPerWarp + q) * 32 + lane, wrow[q] + (size_t)(lane + 32 * nx) * kChunk);
      }
      cp_async_commit();
      cp_async_wait<S - 1>();  // chunk it has landed
      uint4 wv[kRowsPerWarp];
#pragma unroll
      for (int q = 0; q < kRowsPerWarp; ++q) wv[q] = ring[((it % S) * kRowsPerWarp + q) * 32 + lane];
      const int c = lane + 32 * it;
      const int kb = c / (kBlock / kChunk);
      float part[kRowsPerWarp][MR];
#pragma unroll
      for (int q = 0; q < kRowsPerWarp; ++q) {
        float f[kChunk];
        e4m3x16_to_f(wv[q], f);
        float pe[MR], po[MR];  // even / odd elements, two per packed FMA
#pragma unroll
        for (int r = 0; r < MR; ++r) pe[r] = po[r] = 0.f;
#pragma unroll
        for (int e = 0; e < kChunk; e += 2)
#pragma unroll
          for (int r = 0; r < MR; ++r)
            ffma2_vv(pe[r], po[r], f[e], f[e + 1], sA[((size_t)r * kChunk + e) * NC + c],
                     sA[((size_t)r * kChunk + e + 1) * NC + c]);
#pragma unroll
        for (int r = 0; r < MR; ++r) part[q][r] = pe[r] + po[r];
      }
#pragma unroll
      for (int q = 0; q < kRowsPerWarp; ++q) {
        const float ws = __ldg(wsc[q] + kb);
#pragma unroll
        for (int r = 0; r < MR; ++r) acc[q][r] = fmaf(part[q][r], sS[r * KB + kb] * ws, acc[q][r]);
      }
    }
    cp_async_wait<0>();
#pragma unroll
    for (int q = 0; q < kRowsPerWarp; ++q)
#pragma unroll
      for (int r = 0; r < MR; ++r) acc[q][r] = warp_sum(acc[q][r]);
    if (lane < 2 * MR) {  // lane = (column j0 + (lane & 1), row lane >> 1)
      const int jj = lane & 1, r = lane >> 1;
      float gate = 0.f, up = 0.f;
#pragma unroll
      for (int rr = 0; rr < MR; ++rr)
        if (rr == r) {
          gate = jj ? acc[1][rr] : acc[0][rr];
          up = jj ? acc[3][rr] : acc[2][rr];
        }
      if (r < rows) inter[(size_t)(row0 + r) * I + j0 + jj] = up * sm100::rcp_approx(1.0f + __expf(-up)) * gate;
    }
  }
}

// GEMM2 + routing weight.  Unit = (tile, 64 output columns h); warp w takes
// h0 + 4w .. h0 + 4w + 3.
template <int MR>
__global__ void __launch_bounds__(kDecThreads, 1) decode_gemm2_kernel(Gemm2Args a, const float* __restrict__ inter) {
  extern __shared__ float smem[];
  const int H = a.H, I = a.I, KB = I / kBlock, NC = I / kChunk;
  float* sC = smem;  // [MR][16][NC]
  constexpr int S = 4;
  uint4* ring = reinterpret_cast<uint4*>(smem + (size_t)MR * I) + (size_t)(threadIdx.x >> 5) * S * kRowsPerWarp * 32;
  const int num_tiles = min(*a.g.num_tiles, a.g.max_tiles);
  const int per_tile = H / (kRowsPerWarp * kDecWarps);
  int u0, u1;
  unit_range(num_tiles * per_tile, u0, u1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int staged = -1;
  for (int u = u0; u < u1; ++u) {
    const int tile = u / per_tile, hc = u - tile * per_tile;
    const int g = a.g.tile_group[tile], row0 = a.g.tile_row0[tile], rows = min(a.g.tile_rows[tile], MR);
    if (tile != staged) {
      __syncthreads();
      for (int i = threadIdx.x; i < MR * NC; i += blockDim.x) {  // thread per (row, 16-column chunk)
        const int r = i / NC, c = i - r * NC;
#pragma unroll
        for (int q = 0; q < kChunk / 4; ++q) {  // consecutive c: conflict-free stores
          const float4 v = r < rows
                               ? reinterpret_cast<const float4*>(inter + (size_t)(row0 + r) * I + (size_t)c * kChunk)[q]
                               : make_float4(0.f, 0.f, 0.f, 0.f);
          sC[((size_t)r * kChunk + 4 * q) * NC + c] = v.x;
          sC[((size_t)r * kChunk + 4 * q + 1) * NC + c] = v.y;
          sC[((size_t)r * kChunk + 4 * q + 2) * NC + c] = v.z;
          sC[((size_t)r * kChunk + 4 * q + 3) * NC + c] = v.w;
        }
      }
      __syncthreads();
      staged = tile;
    }
    const bool sh = g == a.g.shared_group;
    const uint8_t* W = sh ? a.sw2 : a.w2 + (size_t)g * H * I;
    const float* WS = sh ? a.sw2_scale : a.w2_scale + (size_t)g * (H / kBlock) * KB;
    const int h0 = hc * kRowsPerWarp * kDecWarps + kRowsPerWarp * warp;
    float acc[kRowsPerWarp][MR];
#pragma unroll
    for (int q = 0; q < kRowsPerWarp; ++q)
#pragma unroll
      for (int r = 0; r < MR; ++r) acc[q][r] = 0.f;
    const int n_it = (NC - lane + 31) / 32;
#pragma unroll
    for (int st = 0; st < S - 1; ++st) {
      if (st < n_it) {
#pragma unroll
        for (int q = 0; q < kRowsPerWarp; ++q)
          cp_async16(ring + (st * kRowsPerWarp + q) * 32 + lane,
                     W + (size_t)(h0 + q) * I + (size_t)(lane + 32 * st) * kChunk);
      }
      cp_async_commit();
    }
    for (int it = 0; it < n_it; ++it) {
      const int nx = it + S - 1;
      if (nx < n_it) {
#pragma unroll
        for (int q = 0; q < kRowsPerWarp; ++q)
          cp_async16(ring + ((nx % S) * kRowsPerWarp + q) * 32 + lane,
                     W + (size_t)(h0 + q) * I + (size_t)(lane + 32 * nx) * kChunk);
      }
      cp_async_commit();
      cp_async_wait<S - 1>();
      uint4 wv[kRowsPerWarp];
#pragma unroll
      for (int q = 0; q < kRowsPerWarp; ++q) wv[q] = ring[((it % S) * kRowsPerWarp + q) * 32 + lane];
      const int c = lane + 32 * it;
      const int kb = c / (kBlock / kChunk);
#pragma unroll
      for (int q = 0; q < kRowsPerWarp; ++q) {
        float f[kChunk];
        e4m3x16_to_f(wv[q], f);
        float part[MR], pe[MR], po[MR];
#pragma unroll
        for (int r = 0; r < MR; ++r) pe[r] = po[r] = 0.f;
#pragma unroll
        for (int e = 0; e < kChunk; e += 2)
#pragma unroll
          for (int r = 0; r < MR; ++r)
            ffma2_vv(pe[r], po[r], f[e], f[e + 1], sC[((size_t)r * kChunk + e) * NC + c],
                     sC[((size_t)r * kChunk + e + 1) * NC + c]);
#pragma unroll
        for (int r = 0; r < MR; ++r) part[r] = pe[r] + po[r];
        const float ws = __ldg(WS + (size_t)((h0 + q) / kBlock) * KB + kb);
#pragma unroll
        for (int r = 0; r < MR; ++r) acc[q][r] = fmaf(part[r], ws, acc[q][r]);
      }
    }
    cp_async_wait<0>();
#pragma unroll
    for (int q = 0; q < kRowsPerWarp; ++q)
#pragma unroll
      for (int r = 0; r < MR; ++r) acc[q][r] = warp_sum(acc[q][r]);
    if (lane < kRowsPerWarp * MR) {  // lane = (column h0 + (lane % 4), row lane / 4)
      const int q = lane % kRowsPerWarp, r = lane / kRowsPerWarp;
      float v = 0.f;
#pragma unroll
      for (int qq = 0; qq < kRowsPerWarp; ++qq)
#pragma unroll
        for (int rr = 0; rr < MR; ++rr)
          if (qq == q && rr == r) v = acc[qq][rr];
      if (r < rows) {
        const int row = row0 + r;
        v *= a.row_weight[row];
        if (a.pair_out)
          a.pair_out[(size_t)row * H + h0 + q] = v;
        else
          atomicAdd(a.out + (size_t)a.row_dest[row] * H + h0 + q, v);
      }
    }
  }
}

// Dynamic shared memory above 48 KB needs a per-device opt-in per kernel; the
// bound is the largest size shape_ok admits.
constexpr int kDecSmemMax = 227 * 1024;

template <class K>
int allow_smem(K kernel, std::atomic<uint32_t>& done) {
  int dev = 0;
  GEMMS_CUDA_TRY(cudaGetDevice(&dev));
  const uint32_t bit = 1u << (dev & 31);
  if (!(done.load() & bit)) {
    GEMMS_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kDecSmemMax));
    done.fetch_or(bit);
  }
  return GEMMS_OK;
}

template <int MR>
int launch_gemm1_mr(const Gemm1Args& g1, float* inter, const DecodeSrc& src, cudaStream_t s) {
  static std::atomic<uint32_t> done{0};
  const size_t smem = ((sizeof(float) * ((size_t)MR * g1.H + (size_t)MR * (g1.H / kBlock)) + 15) & ~(size_t)15) +
                      ring_bytes(ring_stages<MR>());
  int rc;
  if ((rc = allow_smem(decode_gemm1_kernel<MR>, done))) return rc;
  // one CTA of 16 warps per SM, each lane keeping S - 1 chunks of four weight
  // rows in flight through its ring
  decode_gemm1_kernel<MR><<<num_sms(), kDecThreads, smem, s>>>(g1, inter, src);
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}

template <int MR>
int launch_gemm2_mr(const Gemm2Args& g2, const float* inter, cudaStream_t s) {
  static std::atomic<uint32_t> done{0};
  const size_t smem = sizeof(float) * (size_t)MR * g2.I + ring_bytes(4);
  int rc;
  if ((rc = allow_smem(decode_gemm2_kernel<MR>, done))) return rc;
  decode_gemm2_kernel<MR><<<num_sms(), kDecThreads, smem, s>>>(g2, inter);
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}

int shape_ok(int H, int I) {
  return H % (kRowsPerWarp * kDecWarps) == 0 && I % (2 * kDecWarps) == 0 && H % kBlock == 0 && I % kBlock == 0 &&
         (size_t)kDecodeMaxRows * (H + H / kBlock) * sizeof(float) + 16 + ring_bytes(ring_stages<kDecodeMaxRows>()) <=
             (size_t)kDecSmemMax &&
         (size_t)2 * (H + H / kBlock) * sizeof(float) + 16 + ring_bytes(ring_stages<2>()) <= (size_t)kDecSmemMax &&
         (size_t)kDecodeMaxRows * I * sizeof(float) + ring_bytes(4) <= (size_t)kDecSmemMax;
}

}  // namespace

int launch_decode_gemm1(const Gemm1Args& g1, float* inter, int max_rows, const DecodeSrc* src, cudaStream_t s) {
  if (max_rows < 1 || max_rows > kDecodeMaxRows || !shape_ok(g1.H, g1.I)) return GEMMS_ERR_SHAPE;
  const DecodeSrc none{};
  const DecodeSrc& sr = src ? *src : none;
  if (sr.row_token && !sr.x_bf16 && !(sr.x_fp8 && sr.x_scale)) return GEMMS_ERR_ARG;
  if (max_rows == 1) return launch_gemm1_mr<1>(g1, inter, sr, s);
  return launch_gemm1_mr<2>(g1, inter, sr, s);
}

int launch_decode_gemm2(const Gemm2Args& g2, const float* inter, int max_rows, cudaStream_t s) {
  if (max_rows < 1 || max_rows > kDecodeMaxRows || !shape_ok(g2.H, g2.I)) return GEMMS_ERR_SHAPE;
  if (max_rows == 1) return launch_gemm2_mr<1>(g2, inter, s);
  return launch_gemm2_mr<2>(g2, inter, s);
}

bool decode_shape_ok(int H, int I) { return shape_ok(H, I); }

}  // namespace gemms
