// router_gemm.cu -- router logits = x . router_w^T on tcgen05 tensor cores.
//
// The reference takes the fp32 logits as an input (flashinfer_baseline.py:6,
// 96); the layer surface moe(x, router_w, ...) computes them here.  x is bf16
// [T, H] and router_w fp32 [E, H].  router_w is split once per call into two
// bf16 planes, hi = bf16(w) and lo = bf16(w - hi) (16 significant bits
// together, relative residual <= 2^-16), and both products accumulate into one
// fp32 TMEM accumulator: x . hi^T + x . lo^T, with exact bf16 x bf16 products.
//
// Work split: one CTA per (128-token M tile, K range).  With few M tiles the K
// dimension is split so that about one CTA per SM runs; each CTA writes its
// fp32 partial [128 x E] to partials[split][t][e] and route_kernel sums the
// splits in a fixed order (deterministic, no atomics).
//
// Decode-sized batches (T <= 128) take a CUDA-core path instead: fp32 FMAs
// over x (bf16, exact in fp32) and router_w read once in fp32, so no bf16
// weight planes are needed; the same split-K partials and fixed-order sum.
//
// CTA: 128 threads.  Thread 0 issues TMA loads of the x tile [128 x 64 bf16]
// and both weight planes [N x 64 bf16] (128-byte swizzle) into a 2-stage ring;
// warp 1 allocates TMEM and one of its threads issues tcgen05.mma.kind::f16
// (M=128, N=E rounded up to 16, K=16); after the last K block all four warps
// read their 32 TMEM lanes and store the partial rows.  Every wait is bounded
// and reports through the error word, like the grouped GEMMs.
#include "common.cuh"
#include "sm100.cuh"

#include <algorithm>
#include <atomic>
#include <cudaTypedefs.h>

namespace gemms {
namespace {
using namespace sm100;

constexpr int RBM = 128;                // tokens per tile (TMEM lanes)
constexpr int RBK = 64;                 // bf16 elements per K block = 128 bytes
constexpr int kStages = 2;
constexpr int kThreads = 128;
constexpr int kSplitTarget = 148;       // B200 SM count: aim at one CTA per SM
constexpr int kSimtMaxT = 128;          // decode-sized batches: CUDA-core fp32 path
constexpr int kSimtExperts = 16;        // experts per CTA (two per warp)

__host__ __device__ inline int pad16(int e) { return (e + 15) / 16 * 16; }

// Instruction descriptor, kind::f16: D fp32, A and B bf16, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// router_w fp32 [E, H] -> planes bf16 [2][Np][H]: hi rows [0, Np), lo rows
// [Np, 2Np); rows >= E of each plane are zero (MMA N is padded to 16).
__global__ void router_split_kernel(const float* __restrict__ w, __nv_bfloat16* __restrict__ planes, int E, int Np,
                                    int H) {
  const size_t per_plane = (size_t)Np * H;
  const size_t n4 = per_plane / 4;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    const size_t o = 4 * i;
    const int row = static_cast<int>(o / H);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (row < E) v = *reinterpret_cast<const float4*>(w + o);
    const __nv_bfloat162 h0 = __floats2bfloat162_rn(v.x, v.y), h1 = __floats2bfloat162_rn(v.z, v.w);
    const float2 b0 = __bfloat1622float2(h0), b1 = __bfloat1622float2(h1);
    const __nv_bfloat162 l0 = __floats2bfloat162_rn(v.x - b0.x, v.y - b0.y);
    const __nv_bfloat162 l1 = __floats2bfloat162_rn(v.z - b1.x, v.w - b1.y);
    uint2 hv, lv;
    hv.x = *reinterpret_cast<const uint32_t*>(&h0);
    hv.y = *reinterpret_cast<const uint32_t*>(&h1);
    lv.x = *reinterpret_cast<const uint32_t*>(&l0);
    lv.y = *reinterpret_cast<const uint32_t*>(&l1);
    *reinterpret_cast<uint2*>(planes + o) = hv;
    *reinterpret_cast<uint2*>(planes + per_plane + o) = lv;
  }
}

// (a0, a1) += (x0, x1) * (w0, w1), one packed fp32x2 FMA.
__device__ __forceinline__ void ffma2v(float& a0, float& a1, float x0, float x1, float w0, float w1) {
  asm("{\n\t.reg .b64 acc, xv, wv;\n\t"
      "mov.b64 acc, {%0, %1};\n\t"
      "mov.b64 xv, {%2, %3};\n\t"
      "mov.b64 wv, {%4, %5};\n\t"
      "fma.rn.f32x2 acc, xv, wv, acc;\n\t"
      "mov.b64 {%0, %1}, acc;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(x0), "f"(x1), "f"(w0), "f"(w1));
}

// Decode path: CTA = 8 warps = 16 experts (two per warp), split = K chunk of
// KC elements; every lane owns KC/32 consecutive columns of both experts' fp32
// rows in registers and streams the T tokens' bf16 columns past them.  Sums
// per lane in a fixed order, then a butterfly over the warp: deterministic.
template <int KC>
__global__ void __launch_bounds__(256) router_simt_kernel(const __nv_bfloat16* __restrict__ x,
                                                          const float* __restrict__ w, int T, int H, int E,
                                                          float* __restrict__ partials) {
  constexpr int PER = KC / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e0 = blockIdx.x * kSimtExperts + 2 * warp;
  const int split = blockIdx.y;
  const int k0 = split * KC + lane * PER;
  float wa[PER], wb[PER];
#pragma unroll
  for (int j = 0; j < PER; j += 4) {
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
    if (e0 < E) a = __ldg(reinterpret_cast<const float4*>(w + (size_t)e0 * H + k0 + j));
    if (e0 + 1 < E) b = __ldg(reinterpret_cast<const float4*>(w + (size_t)(e0 + 1) * H + k0 + j));
    wa[j] = a.x; wa[j + 1] = a.y; wa[j + 2] = a.z; wa[j + 3] = a.w;
    wb[j] = b.x; wb[j + 1] = b.y; wb[j + 2] = b.z; wb[j + 3] = b.w;
  }
  for (int t = 0; t < T; ++t) {
    const uint4* xp = reinterpret_cast<const uint4*>(x + (size_t)t * H + k0);
    float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
#pragma unroll
    for (int j = 0; j < PER; j += 8) {
      const uint4 raw = __ldg(xp + j / 8);
      const uint32_t u[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 xv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[q]));
        ffma2v(a0, a1, xv.x, xv.y, wa[j + 2 * q], wa[j + 2 * q + 1]);
        ffma2v(b0, b1, xv.x, xv.y, wb[j + 2 * q], wb[j + 2 * q + 1]);
      }
    }
    float sa = a0 + a1, sb = b0 + b1;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      sa += __shfl_xor_sync(0xffffffffu, sa, off);
      sb += __shfl_xor_sync(0xffffffffu, sb, off);
    }
    if (lane == 0) {
      float* dst = partials + ((size_t)split * T + t) * E;
      if (e0 < E) dst[e0] = sa;
      if (e0 + 1 < E) dst[e0 + 1] = sb;
    }
  }
}

int simt_chunk(int H) { return H % 1024 == 0 ? 1024 : (H % 512 == 0 ? 512 : 256); }

struct RouterParams {
  int T, E, Np, KB, kb_per_split;
  uint32_t tmem_cols;
  float* partials;  // [splits][T][E]
  int* err;
};

__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() - t0 > GEMMS_WAIT_TIMEOUT_NS) return;
}

__global__ void __launch_bounds__(kThreads, 1)
    router_gemm_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                       const RouterParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tileX = RBM * RBK * 2;          // 16 KB
  const int tileW = p.Np * RBK * 2;         // Np x 128 B per plane
  const int stage = tileX + 2 * tileW;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * stage);
  uint64_t* empty = full + kStages;
  uint64_t* done = empty + kStages;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * RBM;
  const int split = blockIdx.y;
  const int kb0 = split * p.kb_per_split;
  const int nkb = min(p.KB, kb0 + p.kb_per_split) - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, p.tmem_cols);
    tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (threadIdx.x == 0) {
    // ---------------------------------------------------------- producer
    const uint64_t pol = policy_evict_last();  // x tiles and weights are re-read by other CTAs
    int i = 0;
    for (; i < nkb; ++i) {
      const int s = i % kStages;
      if (!mbar_wait(&empty[s], ((i / kStages) & 1) ^ 1, abort_flag, p.err, kErrGemmProducerWait)) break;
      uint8_t* st = smem + s * stage;
      mbar_arrive_expect_tx(&full[s], stage);
      const int kx = (kb0 + i) * RBK;
      tma_load_2d(st, &tmX, &full[s], kx, m0, pol);
      tma_load_2d(st + tileX, &tmW, &full[s], kx, 0, pol);
      tma_load_2d(st + tileX + tileW, &tmW, &full[s], kx, p.Np, pol);
    }
    for (int s = 0; s < kStages && s < i; ++s) {
      const int last = s + kStages * ((i - 1 - s) / kStages);
      drain_wait(&full[s], (last / kStages) & 1);
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------- MMA issuer
    const uint32_t idesc = idesc_bf16_f32(RBM, p.Np);
    const uint32_t d = *reinterpret_cast<volatile const uint32_t*>(tmem_holder);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % kStages;
      if (!mbar_wait(&full[s], (i / kStages) & 1, abort_flag, p.err, kErrGemmMmaWait)) break;
      tc_fence_after();
      uint8_t* st = smem + s * stage;
      const uint64_t ax = smem_desc_k_sw128(smem_u32(st));
      const uint64_t bh = smem_desc_k_sw128(smem_u32(st + tileX));
      const uint64_t bl = smem_desc_k_sw128(smem_u32(st + tileX + tileW));
#pragma unroll
      for (int ks = 0; ks < RBK / 16; ++ks) {  // K = 16 bf16 = 32 bytes = +2 in the start-address field
        umma_bf16(d, ax + 2 * ks, bh + 2 * ks, idesc, (i | ks) != 0);
        umma_bf16(d, ax + 2 * ks, bl + 2 * ks, idesc, 1);
      }
      umma_commit(&empty[s]);
    }
    umma_commit(done);  // also on an abort: lets the epilogue and teardown see issued MMAs finish
  }

  // ---------------------------------------------------------- epilogue
  __syncwarp();
  int got = 1;
  if (lane == 0) {
    got = mbar_wait(done, 0, abort_flag, p.err, kErrGemmEpilogueWait);
    if (!got) drain_wait(done, 0);
  }
  got = __shfl_sync(0xffffffffu, got, 0);
  tc_fence_after();
  const int t = m0 + warp * 32 + lane;
  if (got && !*abort_flag) {
    const uint32_t base = *reinterpret_cast<volatile const uint32_t*>(tmem_holder) +
                          (static_cast<uint32_t>(warp * 32) << 16);
    float* dst = p.partials + ((size_t)split * p.T + t) * p.E;
    for (int c0 = 0; c0 < p.Np; c0 += 32) {
      float v[32];
      tmem_ld_32x32b_x32(base + c0, v);
      tmem_ld_wait();
      if (t < p.T) {
        const int n = min(32, p.E - c0);
        if (n == 32 && (p.E & 3) == 0) {
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(dst + c0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < n) dst[c0 + j] = v[j];
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(*reinterpret_cast<volatile const uint32_t*>(tmem_holder), p.tmem_cols);
  }
}

int make_map_bf16(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return GEMMS_ERR_DRIVER;
  if (!aligned16(base) || (inner * 2) % 16) return GEMMS_ERR_ALIGN;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {inner * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(RBK), box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? GEMMS_OK : GEMMS_ERR_DRIVER;
}

uint32_t tmem_cols_for(int n) {
  uint32_t c = 32;
  while (c < static_cast<uint32_t>(n)) c <<= 1;
  return c;
}

}  // namespace

RouterPlan router_plan(int T, int H, int E) {
  RouterPlan r{};
  if (T <= kSimtMaxT && H % 256 == 0) {  // CUDA-core path: no weight planes
    r.simt = 1;
    r.KB = H / simt_chunk(H);
    r.kb_per_split = 1;
    r.splits = r.KB;
    r.split_bytes = 0;
    r.partial_bytes = align_up(sizeof(float) * (size_t)r.splits * std::max(T, 1) * E, 256);
    return r;
  }
  r.Np = pad16(E);
  r.KB = H / RBK;
  const int m_tiles = std::max(1, cdiv(T, RBM));
  int splits = std::max(1, std::min({kSplitTarget / m_tiles, 32, r.KB}));
  r.kb_per_split = cdiv(r.KB, splits);
  r.splits = cdiv(r.KB, r.kb_per_split);
  r.split_bytes = align_up(sizeof(__nv_bfloat16) * 2 * (size_t)r.Np * H, 256);
  r.partial_bytes = align_up(sizeof(float) * (size_t)r.splits * std::max(T, 1) * E, 256);
  return r;
}

int launch_router_gemm(const RouterGemmArgs& a, cudaStream_t s) {
  if (a.T <= 0) return GEMMS_OK;
  if (a.H % RBK || a.E < 1 || a.E > 256) return GEMMS_ERR_SHAPE;
  const RouterPlan& r = a.plan;
  if (r.simt) {
    if (!aligned16(a.x) || !aligned16(a.router_w) || (a.H % 8)) return GEMMS_ERR_ALIGN;
    const dim3 grid(cdiv(a.E, kSimtExperts), r.splits);
    const int kc = simt_chunk(a.H);
    if (kc == 1024)
      router_simt_kernel<1024><<<grid, 256, 0, s>>>(a.x, a.router_w, a.T, a.H, a.E, a.partials);
    else if (kc == 512)
      router_simt_kernel<512><<<grid, 256, 0, s>>>(a.x, a.router_w, a.T, a.H, a.E, a.partials);
    else
      router_simt_kernel<256><<<grid, 256, 0, s>>>(a.x, a.router_w, a.T, a.H, a.E, a.partials);
    GEMMS_CUDA_TRY(cudaGetLastError());
    return GEMMS_OK;
  }
  if (!aligned16(a.x) || !aligned16(a.router_w) || !aligned16(a.planes) || !aligned16(a.partials))
    return GEMMS_ERR_ALIGN;
  const int nsplit = static_cast<int>(std::min<size_t>(((size_t)r.Np * a.H / 4 + 255) / 256, (size_t)num_sms() * 4));
  router_split_kernel<<<nsplit, 256, 0, s>>>(a.router_w, a.planes, a.E, r.Np, a.H);
  GEMMS_CUDA_TRY(cudaGetLastError());

  CUtensorMap mx, mw;
  int rc;
  if ((rc = make_map_bf16(&mx, a.x, a.H, a.T, RBM))) return rc;
  if ((rc = make_map_bf16(&mw, a.planes, a.H, 2ull * r.Np, r.Np))) return rc;
  RouterParams p{};
  p.T = a.T;
  p.E = a.E;
  p.Np = r.Np;
  p.KB = r.KB;
  p.kb_per_split = r.kb_per_split;
  p.tmem_cols = tmem_cols_for(r.Np);
  p.partials = a.partials;
  p.err = a.err;
  const int smem = kStages * (RBM * RBK * 2 + 2 * r.Np * RBK * 2) + 256 + 1024;
  static std::atomic<unsigned long long> attr_set{0};
  int dev = 0;
  GEMMS_CUDA_TRY(cudaGetDevice(&dev));
  const unsigned long long bit = dev < 64 ? (1ull << dev) : 0ull;
  if (!bit || !(attr_set.load(std::memory_order_relaxed) & bit)) {
    // sized for the largest N (E = 256)
    const int smem_max = kStages * (RBM * RBK * 2 + 2 * 256 * RBK * 2) + 256 + 1024;
    GEMMS_CUDA_TRY(cudaFuncSetAttribute(router_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_max));
    attr_set.fetch_or(bit, std::memory_order_relaxed);
  }
  dim3 grid(cdiv(a.T, RBM), r.splits);
  router_gemm_kernel<<<grid, kThreads, smem, s>>>(mx, mw, p);
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}

}  // namespace gemms

using namespace gemms;

extern "C" size_t gemms_router_workspace_size(int32_t T, int32_t H, int32_t E) {
  if (T < 0 || H <= 0 || H % RBK || E < 1 || E > 256) return 0;
  const RouterPlan r = router_plan(T, H, E);
  return 256 + r.split_bytes + r.partial_bytes;
}

extern "C" int gemms_router_logits(const void* x_bf16, const float* router_w, int32_t T, int32_t H, int32_t E,
                                   float* logits, void* workspace, size_t ws_bytes, gemms_stream_t stream_) {
  if (T < 0 || H <= 0 || H % RBK || E < 1 || E > 256) return GEMMS_ERR_SHAPE;
  if (!x_bf16 || !router_w || !logits) return GEMMS_ERR_ARG;
  const size_t need = gemms_router_workspace_size(T, H, E);
  if (!workspace || ws_bytes < need) return GEMMS_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 255u) return GEMMS_ERR_ALIGN;
  if (T == 0) return GEMMS_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
  char* ws = static_cast<char*>(workspace);
  RouterGemmArgs a{};
  a.plan = router_plan(T, H, E);
  a.x = static_cast<const __nv_bfloat16*>(x_bf16);
  a.router_w = router_w;
  a.T = T;
  a.H = H;
  a.E = E;
  a.err = reinterpret_cast<int*>(ws);
  a.planes = a.plan.split_bytes ? reinterpret_cast<__nv_bfloat16*>(ws + 256) : nullptr;
  a.partials = reinterpret_cast<float*>(ws + 256 + a.plan.split_bytes);
  GEMMS_CUDA_TRY(cudaMemsetAsync(ws, 0, 256, st));
  int rc = launch_router_gemm(a, st);
  if (rc) return rc;
  return launch_sum_partials(a.partials, a.plan.splits, T, E, logits, st);
}
