// ep.cu -- expert-parallel dispatch / receive-side expert FFN / combine.
//
// The reference has no distributed path: its only hook is local_expert_offset
// (flashinfer_baseline.py:132-138, persistent_kernel2.cu:332).  Rank r owns
// experts [r*E_local, (r+1)*E_local); these kernels build the exchange around
// that convention (the all-to-alls themselves are NCCL calls issued by the
// host, gemms_b200/ep.py):
//
//   dispatch  : per token, the set of destination ranks holding any of its
//               top-k experts (each token goes once to each such rank); rows
//               are laid out grouped by destination in increasing token order
//               (deterministic).  The token is quantised per 1x128 once and
//               packed with its scales and the ids/weights of the experts
//               that live on the destination.  Also writes the token-major
//               quantised rows used by the local shared expert.
//   expert ffn: the packed received rows, read in place (strided), go through
//               histogram -> plan -> assign -> permute -> GEMM1 -> GEMM2; each
//               received row's result is pre-reduced over its local experts in
//               fp32.
//   pack back : each pre-reduced fp32 row is sent back as fp16 values divided
//               by a per-row power of two 2^e (max|row| / 2^e < 2^15), so the
//               scaling is exact and the only new rounding is fp16's (2^-11
//               relative, below the output's bf16 rounding); halves the bytes
//               of the combine all-to-all.
//   combine   : out[t] = bf16(acc[t] + sum over t's destinations of the rows
//               sent back), gathered deterministically.
//
// Packed row layout (row_bytes = align16(H + 4*H/128 + 8*top_k)):
//   [0, H)                    e4m3 activations
//   [H, H + 4*H/128)          fp32 1x128 scales
//   [.., + 4*top_k)           int32 global expert ids on the destination, -1 padded
//   [.., + 4*top_k)           fp32 routing weights
// Packed combine row (back_row_bytes = align16(2*H + 4)):
//   [0, 2H)                   fp16 values / 2^e
//   [2H, 2H + 4)              fp32 2^e
#include "common.cuh"
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>

namespace gemms {
namespace {

constexpr int kMaxWorld = 32;

__host__ __device__ inline size_t ep_row_bytes(int H, int top_k) {
  return align_up((size_t)H + 4 * (size_t)(H / kBlock) + 8 * (size_t)top_k, 16);
}

__host__ __device__ inline size_t ep_back_row_bytes(int H) { return align_up(2 * (size_t)H + 4, 16); }

__device__ __forceinline__ unsigned dest_mask(const int32_t* idx, int top_k, int E_local) {
  unsigned m = 0;
  for (int j = 0; j < top_k; ++j) {
    const int e = idx[j];
    if (e >= 0) m |= 1u << (e / E_local);
  }
  return m;
}

// Per-destination row counts (send_counts[0][d]) and routed (token, expert)
// pairs (send_counts[1][d]), which size the destination's grouped rows
// exactly.  Thread per token; the counts are summed per warp
// (__reduce_add_sync), then per block in shared memory, and each block adds
// its 2 x world totals with one global atomic each (per-token atomics onto the
// same few counters serialise in L2).
__global__ void __launch_bounds__(256) ep_count_kernel(const int32_t* __restrict__ topk_idx, int T, int top_k,
                                                       int E_local, int world, int32_t* __restrict__ send_counts) {
  __shared__ int s_cnt[2 * kMaxWorld];
  const int tid = threadIdx.x, lane = tid & 31;
  if (tid < 2 * world) s_cnt[tid] = 0;
  __syncthreads();
  const int stride = gridDim.x * blockDim.x;
  for (int t0 = blockIdx.x * blockDim.x; t0 < T; t0 += stride) {  // block-uniform trip count
    const int t = t0 + tid;
    const int32_t* idx = topk_idx + (size_t)t * top_k;
    const unsigned m = t < T ? dest_mask(idx, top_k, E_local) : 0u;
    for (int d = 0; d < world; ++d) {
      int pairs = 0;
      if ((m >> d) & 1u)
        for (int j = 0; j < top_k; ++j) pairs += (idx[j] >= 0 && idx[j] / E_local == d);
      const unsigned rows_w = __reduce_add_sync(0xffffffffu, (m >> d) & 1u);
      const unsigned pairs_w = __reduce_add_sync(0xffffffffu, static_cast<unsigned>(pairs));
      if (lane == 0 && rows_w) {
        atomicAdd(&s_cnt[d], static_cast<int>(rows_w));
        atomicAdd(&s_cnt[world + d], static_cast<int>(pairs_w));
      }
    }
  }
  __syncthreads();
  if (tid < 2 * world && s_cnt[tid]) atomicAdd(send_counts + tid, s_cnt[tid]);
}

// Block per destination: send rows in increasing token order.
__global__ void __launch_bounds__(1024) ep_assign_kernel(const int32_t* __restrict__ topk_idx, int T, int top_k,
                                                         int E_local, int world,
                                                         const int32_t* __restrict__ send_counts,
                                                         int32_t* __restrict__ send_row_of) {
  __shared__ int s_warp[32];
  __shared__ int s_base;
  const int d = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  if (tid == 0) {
    int o = 0;
    for (int i = 0; i < d; ++i) o += send_counts[i];
    s_base = o;
  }
  __syncthreads();
  for (int t0 = 0; t0 < T; t0 += blockDim.x) {
    const int t = t0 + tid;
    bool f = false;
    if (t < T) f = (dest_mask(topk_idx + (size_t)t * top_k, top_k, E_local) >> d) & 1u;
    const unsigned ballot = __ballot_sync(0xffffffffu, f);
    if (lane == 0) s_warp[warp] = __popc(ballot);
    __syncthreads();
    if (warp == 0) {
      int v = lane < nwarps ? s_warp[lane] : 0;
      for (int off = 1; off < 32; off <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, v, off);
        if (lane >= off) v += o;
      }
      if (lane < nwarps) s_warp[lane] = v;
    }
    __syncthreads();
    const int base = s_base;
    if (t < T) {
      send_row_of[(size_t)t * world + d] =
          f ? base + (warp > 0 ? s_warp[warp - 1] : 0) + __popc(ballot & ((1u << lane) - 1u)) : -1;
    }
    __syncthreads();
    if (tid == 0) s_base = base + s_warp[nwarps - 1];
    __syncthreads();
  }
}

// Block (8 warps) per token: quantise once, write the token-major rows and
// every packed send row of the token.
__global__ void __launch_bounds__(256, 4) ep_pack_kernel(const __nv_bfloat16* __restrict__ x,
                                                      const int32_t* __restrict__ topk_idx,
                                                      const float* __restrict__ topk_w, int T, int H, int top_k,
                                                      int E_local, int world,
                                                      const int32_t* __restrict__ send_row_of,
                                                      uint8_t* __restrict__ send_buf, size_t row_bytes,
                                                      uint8_t* __restrict__ xq, float* __restrict__ xq_scale) {
  __shared__ int s_rows[kMaxWorld];
  __shared__ int s_dests[kMaxWorld];
  __shared__ int s_nd;
  const int t = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (warp == 0) {  // the token's send rows, compacted in destination order
    const int r = lane < world ? send_row_of[(size_t)t * world + lane] : -1;
    const unsigned b = __ballot_sync(0xffffffffu, r >= 0);
    if (r >= 0) {
      const int i = __popc(b & ((1u << lane) - 1u));
      s_rows[i] = r;
      s_dests[i] = lane;
    }
    if (lane == 0) s_nd = __popc(b);
  }
  __syncthreads();
  const int nd = s_nd;
  const int KB = H / kBlock;
  for (int kb = warp; kb < KB; kb += 8) {
    const uint2 raw = *reinterpret_cast<const uint2*>(x + (size_t)t * H + (size_t)kb * kBlock + lane * 4);
    const __nv_bfloat162 p0 = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
    const __nv_bfloat162 p1 = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
    const float v0 = __low2float(p0), v1 = __high2float(p0), v2 = __low2float(p1), v3 = __high2float(p1);
    float amax = fmaxf(fmaxf(fabsf(v0), fabsf(v1)), fmaxf(fabsf(v2), fabsf(v3)));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const float scale = amax > 0.f ? __fdiv_rn(amax, kFp8Max) : 1.0f;
    const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(
        make_float2(__fdiv_rn(v0, scale), __fdiv_rn(v1, scale)), __NV_SATFINITE, __NV_E4M3);
    const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(
        make_float2(__fdiv_rn(v2, scale), __fdiv_rn(v3, scale)), __NV_SATFINITE, __NV_E4M3);
    const uint32_t packed = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
    *reinterpret_cast<uint32_t*>(xq + (size_t)t * H + (size_t)kb * kBlock + lane * 4) = packed;
    if (lane == 0) xq_scale[(size_t)kb * T + t] = scale;
    for (int i = 0; i < nd; ++i) {
      uint8_t* row = send_buf + (size_t)s_rows[i] * row_bytes;
      *reinterpret_cast<uint32_t*>(row + (size_t)kb * kBlock + lane * 4) = packed;
      if (lane == 0) reinterpret_cast<float*>(row + H)[kb] = scale;
    }
  }
  // expert ids / weights that live on each destination
  if (warp == 0) {
    for (int i = 0; i < nd; ++i) {
      uint8_t* row = send_buf + (size_t)s_rows[i] * row_bytes;
      int32_t* ids = reinterpret_cast<int32_t*>(row + H + 4 * KB);
      float* ws = reinterpret_cast<float*>(row + H + 4 * KB + 4 * top_k);
      for (int j = lane; j < top_k; j += 32) {
        const int e = topk_idx[(size_t)t * top_k + j];
        const bool here = e >= 0 && e / E_local == s_dests[i];
        ids[j] = here ? e : -1;
        ws[j] = here ? topk_w[(size_t)t * top_k + j] : 0.f;
      }
    }
  }
}

// Thread per received row (grid-stride): local-expert histogram and
// pair_row = -1.  Counts go to a per-block histogram in shared memory and each
// block adds its non-zero bins to `counts` (experts past the shared bins, if
// E_local ever exceeded them, count with global atomics directly).
constexpr int kEpHistBins = 1024;
__global__ void __launch_bounds__(256) ep_hist_kernel(const uint8_t* __restrict__ recv, size_t row_bytes, int R,
                                                      const int32_t* R_dev, int H, int top_k, int local_offset,
                                                      int E_local, int32_t* __restrict__ counts,
                                                      int32_t* __restrict__ pair_row, int* err) {
  __shared__ int s_hist[kEpHistBins];
  const int bins = min(E_local, kEpHistBins);
  for (int i = threadIdx.x; i < bins; i += blockDim.x) s_hist[i] = 0;
  __syncthreads();
  const int n = R_dev ? min(R, *R_dev) : R;
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < n; r += gridDim.x * blockDim.x) {
    const int32_t* ids = reinterpret_cast<const int32_t*>(recv + (size_t)r * row_bytes + H + 4 * (H / kBlock));
    for (int j = 0; j < top_k; ++j) {
      pair_row[(size_t)r * top_k + j] = -1;
      const int e = ids[j];
      if (e < 0) continue;
      const int le = e - local_offset;
      if (le >= 0 && le < E_local) {
        if (le < bins)
          atomicAdd(&s_hist[le], 1);
        else
          atomicAdd(counts + le, 1);
      } else {
        atomicOr(err, kErrBadExpertIndex);
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < bins; i += blockDim.x)
    if (s_hist[i]) atomicAdd(counts + i, s_hist[i]);
}

// Block per token: out[t] = bf16(acc[t] + sum of the token's returned rows).
// Block per row: amax, then the row's values divided by 2^e as fp16.
__global__ void __launch_bounds__(256) ep_pack_back_kernel(const float* __restrict__ rows, const int32_t* R_dev,
                                                           int H, uint8_t* __restrict__ packed, size_t rbb) {
  __shared__ float s_warp[8];
  const size_t r = blockIdx.x;
  if (R_dev && (int)r >= *R_dev) return;
  const float4* src = reinterpret_cast<const float4*>(rows + r * H);
  float amax = 0.f;
  for (int c = threadIdx.x; c < H / 4; c += blockDim.x) {
    const float4 v = src[c];
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  if ((threadIdx.x & 31) == 0) s_warp[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = s_warp[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) amax = fmaxf(amax, s_warp[w]);
  // amax = m * 2^x with m in [0.5, 1): amax < 2^x, so e = x - 15 keeps every
  // |value| / 2^e below 2^15 (fp16 max 65504).  Zero / non-finite rows: e = 0.
  int x = 0;
  if (amax > 0.f && isfinite(amax)) frexpf(amax, &x), x -= 15;
  uint8_t* dst = packed + r * rbb;
  for (int c = threadIdx.x; c < H / 4; c += blockDim.x) {
    const float4 v = src[c];
    const __half2 lo = __floats2half2_rn(ldexpf(v.x, -x), ldexpf(v.y, -x));
    const __half2 hi = __floats2half2_rn(ldexpf(v.z, -x), ldexpf(v.w, -x));
    uint2 o;
    o.x = *reinterpret_cast<const uint32_t*>(&lo);
    o.y = *reinterpret_cast<const uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(dst + 8 * (size_t)c) = o;
  }
  if (threadIdx.x == 0) *reinterpret_cast<float*>(dst + 2 * (size_t)H) = ldexpf(1.0f, x);
}

// Where each destination's packed combine rows live: row (send_row_of[t, d] +
// add[d]) of the buffer at base[d].  One buffer for the all-to-all path;
// each rank's own buffer (peer pointers, read over NVLink) for the peer path.
struct BackRows {
  const uint8_t* base[kMaxWorld];
  int add[kMaxWorld];
  const int32_t* add_dev;  // when set, add[d] = add_dev[d] (offsets computed on the device)
  int cap;                 // > 0: rows at or past it are outside the buffers and are skipped
};

// out = bf16(acc + rows), or with add_to (acc, out unused): add_to += rows in
// fp32 with one vector atomic per 4 columns (for a sum that other kernels add
// into at the same time, e.g. the shared expert's GEMMs).
__global__ void __launch_bounds__(256) ep_combine_kernel(const float* __restrict__ acc, const BackRows rows_at,
                                                         size_t rbb, const int32_t* __restrict__ send_row_of, int T,
                                                         int H, int world, __nv_bfloat16* __restrict__ out,
                                                         float* __restrict__ add_to) {
  __shared__ const uint8_t* s_rows[kMaxWorld];
  __shared__ float s_scale[kMaxWorld];
  __shared__ int s_nd;
  const int t = blockIdx.x;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x < 32) {  // the token's returned rows, compacted in rank order
    const int d = lane;
    int r = d < world ? send_row_of[(size_t)t * world + d] : -1;
    int add = 0;
    if (r >= 0) {
      add = rows_at.add_dev ? rows_at.add_dev[d] : rows_at.add[d];
      if (rows_at.cap > 0 && (r + add < 0 || r + add >= rows_at.cap)) r = -1;  // not in the buffer: skipped
    }
    const unsigned b = __ballot_sync(0xffffffffu, r >= 0);
    if (r >= 0) {
      const int i = __popc(b & ((1u << lane) - 1u));
      const uint8_t* row = rows_at.base[d] + (size_t)(r + add) * rbb;
      s_rows[i] = row;
      s_scale[i] = *reinterpret_cast<const float*>(row + 2 * (size_t)H);
    }
    if (lane == 0) s_nd = __popc(b);
  }
  __syncthreads();
  const int nd = s_nd;
  const uint8_t* const* rows = s_rows;
  const float* scale = s_scale;
  if (add_to && nd == 0) return;
  for (int c = threadIdx.x * 4; c < H; c += blockDim.x * 4) {
    float4 s = add_to ? make_float4(0.f, 0.f, 0.f, 0.f) : *reinterpret_cast<const float4*>(acc + (size_t)t * H + c);
    for (int i = 0; i < nd; ++i) {
      const uint2 b = *reinterpret_cast<const uint2*>(rows[i] + 2 * (size_t)c);
      const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&b.x));
      const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&b.y));
      s.x = fmaf(lo.x, scale[i], s.x);
      s.y = fmaf(lo.y, scale[i], s.y);
      s.z = fmaf(hi.x, scale[i], s.z);
      s.w = fmaf(hi.y, scale[i], s.w);
    }
    if (add_to) {
      atomicAdd(reinterpret_cast<float4*>(add_to + (size_t)t * H + c), s);
      continue;
    }
    __nv_bfloat162 lo = __floats2bfloat162_rn(s.x, s.y), hi = __floats2bfloat162_rn(s.z, s.w);
    uint2 o;
    o.x = *reinterpret_cast<uint32_t*>(&lo);
    o.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(out + (size_t)t * H + c) = o;
  }
}

// ---- device-driven exchange over symmetric (NVLink-mapped) memory ----------
// Each rank's exchange region, allocated symmetrically so that every rank can
// address every other rank's copy:
//   [0, kEpHdrBytes)            int32 counts [2][world] (gemms_ep_dispatch's send_counts)
//   [kEpHdrBytes, +send_cap*rb) send rows grouped by destination in token order
// The receiving rank reads the counts and then its rows straight out of the
// senders' regions (loads over NVLink): no host read of a count matrix and no
// split sizes on the host.
constexpr size_t kEpHdrBytes = 256;

// CTAs of the row pull (0: two per SM); fewer leave SMs to a GEMM running
// beside it on another stream.
std::atomic<int> g_pull_ctas{0};
int pull_ctas() { return g_pull_ctas.load(); }

// Exchange plan (int32 [kEpInfoInts], device): see gemms_ep_pull in the header.
constexpr int kInfoR = 0, kInfoP = 1, kInfoFlags = 2, kInfoStart = 8, kInfoSrcOff = 48, kInfoAdd = 88;

struct PeerRegions {
  const uint8_t* base[kMaxWorld];
};

__device__ __forceinline__ int ld_sys(const int32_t* p) {
  int v;
  asm volatile("ld.relaxed.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One warp; lane s reads source rank s's counts.  Received rows are ordered by
// source rank, then by the source's token order (the layout an all-to-all
// would produce).  Counts that do not fit the regions (a corrupt or foreign
// header) set a flag and plan no rows, so no load leaves the regions.
__global__ void ep_pull_plan_kernel(PeerRegions reg, int rank, int world, int send_cap, int recv_cap,
                                    int32_t* __restrict__ info) {
  const unsigned full = 0xffffffffu;
  const int s = threadIdx.x;
  const bool live = s < world;
  int rows_to_me = 0, pairs_to_me = 0, my_off = 0, add = 0, flags = 0;
  if (live) {
    const int32_t* hdr = reinterpret_cast<const int32_t*>(reg.base[s]);
    int sent = 0;
    for (int d = 0; d < world; ++d) {
      const int m = ld_sys(hdr + d);
      if (m < 0) flags |= 2;
      if (d < rank) my_off += m;
      if (d == rank) rows_to_me = m;
      sent += m;
    }
    pairs_to_me = ld_sys(hdr + world + rank);
    if (sent > send_cap || pairs_to_me < 0) flags |= 2;
    // lane d as a destination: this rank's rows for d start, in d's receive
    // order, after the rows of ranks q < rank; in this rank's send rows they
    // start after the rows for destinations d' < d.
    const int32_t* mine = reinterpret_cast<const int32_t*>(reg.base[rank]);
    int before = 0, send_off = 0;
    for (int q = 0; q < rank; ++q) before += ld_sys(reinterpret_cast<const int32_t*>(reg.base[q]) + s);
    for (int d = 0; d < s; ++d) send_off += ld_sys(mine + d);
    add = before - send_off;
  }
  int incl = rows_to_me;
  for (int off = 1; off < 32; off <<= 1) {
    const int v = __shfl_up_sync(full, incl, off);
    if (s >= off) incl += v;
  }
  int P = pairs_to_me;
  for (int off = 16; off > 0; off >>= 1) {
    P += __shfl_xor_sync(full, P, off);
    flags |= __shfl_xor_sync(full, flags, off);
  }
  const int total = __shfl_sync(full, incl, 31);
  if (total > recv_cap) flags |= 1;
  const int R = flags ? 0 : total;  // nothing is pulled past a capacity or from bad counts
  if (live) {
    info[kInfoStart + s] = incl - rows_to_me;
    info[kInfoSrcOff + s] = my_off;
    info[kInfoAdd + s] = add;
  }
  if (s == 0) {
    info[kInfoStart + world] = total;
    info[kInfoR] = R;
    info[kInfoP] = flags ? 0 : P;
    info[kInfoFlags] = flags;
  }
}

// Grid-stride over the 16-byte chunks of all received rows: each thread
// issues kPullUnroll loads (from the source rank's region, over NVLink for a
// peer) before its stores, so a CTA keeps 32 KB in flight; consecutive threads
// take consecutive chunks of a row (coalesced on both sides).
constexpr int kPullUnroll = 8;

__global__ void __launch_bounds__(256) ep_pull_rows_kernel(PeerRegions reg, const int32_t* __restrict__ info,
                                                           int world, size_t rb, uint8_t* __restrict__ recv) {
  __shared__ int s_start[kMaxWorld + 1];
  __shared__ int s_off[kMaxWorld];
  if ((int)threadIdx.x <= world) s_start[threadIdx.x] = info[kInfoStart + threadIdx.x];
  if ((int)threadIdx.x < world) s_off[threadIdx.x] = info[kInfoSrcOff + threadIdx.x];
  __syncthreads();
  const int R = info[kInfoR];
  const int n16 = static_cast<int>(rb / 16);
  const long long total = (long long)R * n16;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long base = (long long)blockIdx.x * blockDim.x + threadIdx.x; base < total;
       base += stride * kPullUnroll) {
    uint4 v[kPullUnroll];
    uint4* dst[kPullUnroll];
#pragma unroll
    for (int u = 0; u < kPullUnroll; ++u) {
      const long long i = base + u * stride;
      dst[u] = nullptr;
      if (i < total) {
        const int r = static_cast<int>(i / n16);
        const int c = static_cast<int>(i - (long long)r * n16);
        int s = 0;
        while (s + 1 < world && s_start[s + 1] <= r) ++s;
        const uint4* src = reinterpret_cast<const uint4*>(reg.base[s] + kEpHdrBytes +
                                                          (size_t)(s_off[s] + r - s_start[s]) * rb);
        v[u] = src[c];
        dst[u] = reinterpret_cast<uint4*>(recv + (size_t)r * rb) + c;
      }
    }
#pragma unroll
    for (int u = 0; u < kPullUnroll; ++u)
      if (dst[u]) *dst[u] = v[u];
  }
}

// out[0 : *R_dev rows) = 0 (rows counted on the device).
__global__ void ep_zero_rows_kernel(float4* __restrict__ out, const int32_t* __restrict__ R_dev, int R_cap, int H) {
  const size_t n = (size_t)min(*R_dev, R_cap) * (H / 4);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    out[i] = make_float4(0.f, 0.f, 0.f, 0.f);
}

struct EpFfnLayout {
  int P;  // grouped (received row, local expert) pair rows the buffers hold
  int groups, max_tiles, scale_ld;
  size_t err, counts, offsets, tile_group, tile_row0, tile_rows, num_tiles, pair_row, row_token, row_weight;
  size_t a_rows, a_scale, inter, inter_scale, total, head;
};

EpFfnLayout ep_ffn_layout(int R_max, int P_max, int H, int I, int E_local, int top_k, int planes) {
  EpFfnLayout L{};
  const int P = std::max(std::min(P_max, R_max * top_k), 1);  // grouped pair rows
  L.P = P;
  L.groups = E_local;
  L.max_tiles = cdiv(P, kBlock) + E_local;
  L.scale_ld = static_cast<int>(align_up(P, 32));
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align_up(o + bytes, 256);
    return at;
  };
  L.err = take(64);
  L.counts = take(sizeof(int32_t) * std::max(E_local, 1));
  L.head = o;
  L.offsets = take(sizeof(int32_t) * 2 * (E_local + 1));  // offsets, then first tile per group
  L.tile_group = take(sizeof(int32_t) * L.max_tiles);
  L.tile_row0 = take(sizeof(int32_t) * L.max_tiles);
  L.tile_rows = take(sizeof(int32_t) * L.max_tiles);
  L.num_tiles = take(sizeof(int32_t));
  L.pair_row = take(sizeof(int32_t) * (size_t)std::max(R_max, 1) * top_k);
  L.row_token = take(sizeof(int32_t) * P);
  L.row_weight = take(sizeof(float) * P);
  L.a_rows = take((size_t)P * H);
  L.a_scale = take(sizeof(float) * (size_t)(H / kBlock) * L.scale_ld);
  L.inter = take((size_t)P * planes * I);
  L.inter_scale = take(sizeof(float) * (size_t)(I / kBlock) * L.scale_ld);
  L.total = o;
  return L;
}

template <class T>
T* at(void* ws, size_t off) {
  return reinterpret_cast<T*>(static_cast<char*>(ws) + off);
}

}  // namespace
}  // namespace gemms

using namespace gemms;

extern "C" {

size_t gemms_ep_row_bytes(int32_t H, int32_t top_k) { return ep_row_bytes(H, top_k); }

int gemms_ep_dispatch(const int32_t* topk_idx, const float* topk_w, const void* x_bf16, int32_t T, int32_t H,
                      int32_t top_k, int32_t world, int32_t E_local, int32_t* send_counts, int32_t* send_row_of,
                      void* send_buf, void* xq, float* xq_scale, gemms_stream_t stream_) {
  if (T < 0 || H <= 0 || H % kBlock || top_k < 1 || top_k > 16 || world < 1 || world > kMaxWorld || E_local < 1)
    return GEMMS_ERR_SHAPE;
  if (!topk_idx || !topk_w || !x_bf16 || !send_counts || !send_row_of || !send_buf || !xq || !xq_scale)
    return GEMMS_ERR_ARG;
  if (!aligned16(send_buf) || !aligned16(xq) || !aligned16(x_bf16)) return GEMMS_ERR_ALIGN;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
  GEMMS_CUDA_TRY(cudaMemsetAsync(send_counts, 0, sizeof(int32_t) * 2 * world, st));
  if (T == 0) return GEMMS_OK;
  ep_count_kernel<<<std::max(1, std::min(cdiv(T, 256), num_sms())), 256, 0, st>>>(topk_idx, T, top_k, E_local,
                                                                                   world, send_counts);
  GEMMS_CUDA_TRY(cudaGetLastError());
  ep_assign_kernel<<<world, 1024, 0, st>>>(topk_idx, T, top_k, E_local, world, send_counts, send_row_of);
  GEMMS_CUDA_TRY(cudaGetLastError());
  ep_pack_kernel<<<T, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x_bf16), topk_idx, topk_w, T, H, top_k,
                                     E_local, world, send_row_of, static_cast<uint8_t*>(send_buf),
                                     ep_row_bytes(H, top_k), static_cast<uint8_t*>(xq), xq_scale);
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}

size_t gemms_ep_ffn_workspace_size(int32_t R_max, int32_t P_max, int32_t H, int32_t I, int32_t E_local,
                                   int32_t top_k, int32_t inter_planes) {
  const int planes = inter_planes == 0 ? 2 : inter_planes;
  if (R_max < 0 || P_max < 0 || H <= 0 || I <= 0 || E_local < 1 || H % 256 || I % kBlock || top_k < 1 ||
      top_k > 16 || planes < 2 || planes > 3)
    return 0;
  return ep_ffn_layout(R_max, P_max, H, I, E_local, top_k, planes).total;
}

}  // extern "C"

namespace {

// R rows (R_dev == nullptr) or the first *R_dev of R_cap = R rows.
int ep_expert_ffn_impl(const void* recv_buf, int32_t R, const int32_t* R_dev, int32_t P_max, int32_t H, int32_t I,
                       int32_t top_k, int32_t E_local, int32_t local_expert_offset, int32_t inter_planes,
                       const void* w13, const float* w13_scale, const void* w2, const float* w2_scale,
                       float* out_rows, void* workspace, size_t ws_bytes, gemms_stream_t stream_) {
  const int planes = inter_planes == 0 ? 2 : inter_planes;
  if (R < 0 || P_max < 0 || H <= 0 || I <= 0 || E_local < 1 || H % 256 || I % kBlock || top_k < 1 || top_k > 16 ||
      planes < 2 || planes > 3)
    return GEMMS_ERR_SHAPE;
  if (!recv_buf || !w13 || !w13_scale || !w2 || !w2_scale || !out_rows) return GEMMS_ERR_ARG;
  const EpFfnLayout L = ep_ffn_layout(R, P_max, H, I, E_local, top_k, planes);
  if (!workspace || ws_bytes < L.total) return GEMMS_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 255u) return GEMMS_ERR_ALIGN;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
  if (R == 0) return GEMMS_OK;
  void* ws = workspace;
  int* err = at<int>(ws, L.err);
  const size_t rb = ep_row_bytes(H, top_k);
  const uint8_t* recv = static_cast<const uint8_t*>(recv_buf);
  GEMMS_CUDA_TRY(cudaMemsetAsync(ws, 0, L.head, st));
  if (R_dev) {
    ep_zero_rows_kernel<<<num_sms() * 4, 256, 0, st>>>(reinterpret_cast<float4*>(out_rows), R_dev, R, H);
    GEMMS_CUDA_TRY(cudaGetLastError());
  } else {
    GEMMS_CUDA_TRY(cudaMemsetAsync(out_rows, 0, sizeof(float) * (size_t)R * H, st));
  }
  int32_t* pair_row = at<int32_t>(ws, L.pair_row);
  ep_hist_kernel<<<std::max(1, std::min(cdiv(R, 256), num_sms())), 256, 0, st>>>(
      recv, rb, R, R_dev, H, top_k, local_expert_offset, E_local, at<int32_t>(ws, L.counts), pair_row, err);
  GEMMS_CUDA_TRY(cudaGetLastError());
  int rc;
  PlanArgs pa{};
  pa.counts = at<int32_t>(ws, L.counts);
  pa.E_local = E_local;
  pa.shared_rows = 0;
  pa.offsets = at<int32_t>(ws, L.offsets);
  pa.tile_group = at<int32_t>(ws, L.tile_group);
  pa.tile_row0 = at<int32_t>(ws, L.tile_row0);
  pa.tile_rows = at<int32_t>(ws, L.tile_rows);
  pa.num_tiles = at<int32_t>(ws, L.num_tiles);
  pa.group_tile0 = pa.offsets + (E_local + 1);
  pa.max_tiles = L.max_tiles;
  pa.row_capacity = L.P;
  pa.err = err;
  if ((rc = launch_plan(pa, st))) return rc;

  const int KB = H / kBlock;
  AssignArgs sa{};
  sa.topk_idx = reinterpret_cast<const int32_t*>(recv + H + 4 * KB);
  sa.topk_w = reinterpret_cast<const float*>(recv + H + 4 * KB + 4 * top_k);
  sa.idx_stride = static_cast<int>(rb / 4);
  sa.T = R;
  sa.T_dev = R_dev;
  sa.top_k = top_k;
  sa.local_offset = local_expert_offset;
  sa.E_local = E_local;
  sa.offsets = pa.offsets;
  sa.row_token = at<int32_t>(ws, L.row_token);
  sa.row_weight = at<float>(ws, L.row_weight);
  sa.pair_row = pair_row;
  sa.shared_rows = 0;
  sa.row_capacity = L.P;
  if ((rc = launch_assign(sa, st))) return rc;

  PermuteArgs qa{};
  qa.mode = GEMMS_INPUT_FP8;
  qa.x_fp8 = recv;
  qa.x_scale = reinterpret_cast<const float*>(recv + H);
  qa.x_row_stride = static_cast<long long>(rb);
  qa.scale_kb_stride = 1;
  qa.scale_t_stride = static_cast<long long>(rb / 4);
  qa.T = R;
  qa.T_dev = R_dev;
  qa.H = H;
  qa.top_k = top_k;
  qa.pair_row = pair_row;
  qa.shared_row0 = nullptr;
  qa.rows_fp8 = at<uint8_t>(ws, L.a_rows);
  qa.rows_scale = at<float>(ws, L.a_scale);
  qa.scale_ld = L.scale_ld;
  if ((rc = launch_permute(qa, st))) return rc;

  GemmGroupsArgs gg{};
  gg.tile_group = pa.tile_group;
  gg.tile_row0 = pa.tile_row0;
  gg.tile_rows = pa.tile_rows;
  gg.num_tiles = pa.num_tiles;
  gg.group_tile0 = pa.group_tile0;
  gg.max_tiles = L.max_tiles;
  gg.shared_group = -1;
  const int P = L.P;

  Gemm1Args g1{};
  g1.g = gg;
  g1.a = qa.rows_fp8;
  g1.a_rows = P;
  g1.a_scale = qa.rows_scale;
  g1.a_scale_ld = L.scale_ld;
  g1.w13 = static_cast<const uint8_t*>(w13);
  g1.w13_scale = w13_scale;
  g1.E_local = E_local;
  g1.H = H;
  g1.I = I;
  g1.planes = planes;
  g1.inter = at<uint8_t>(ws, L.inter);
  g1.inter_scale = at<float>(ws, L.inter_scale);
  g1.inter_scale_ld = L.scale_ld;
  g1.err = err;
  if ((rc = launch_gemm1(g1, st))) return rc;

  Gemm2Args g2{};
  g2.g = gg;
  g2.inter = g1.inter;
  g2.a_rows = P;
  g2.inter_scale = g1.inter_scale;
  g2.inter_scale_ld = L.scale_ld;
  g2.w2 = static_cast<const uint8_t*>(w2);
  g2.w2_scale = w2_scale;
  g2.E_local = E_local;
  g2.H = H;
  g2.I = I;
  g2.planes = planes;
  g2.row_dest = sa.row_token;
  g2.row_weight = sa.row_weight;
  g2.out = out_rows;
  g2.err = err;
  return launch_gemm2(g2, st);
}

}  // namespace

extern "C" {

int gemms_ep_expert_ffn(const void* recv_buf, int32_t R, int32_t P_max, int32_t H, int32_t I, int32_t top_k,
                        int32_t E_local, int32_t local_expert_offset, int32_t inter_planes, const void* w13,
                        const float* w13_scale, const void* w2, const float* w2_scale, float* out_rows,
                        void* workspace, size_t ws_bytes, gemms_stream_t stream) {
  return ep_expert_ffn_impl(recv_buf, R, nullptr, P_max, H, I, top_k, E_local, local_expert_offset, inter_planes,
                            w13, w13_scale, w2, w2_scale, out_rows, workspace, ws_bytes, stream);
}

int gemms_ep_expert_ffn_dev(const void* recv_buf, int32_t R_cap, const int32_t* info, int32_t P_max, int32_t H,
                            int32_t I, int32_t top_k, int32_t E_local, int32_t local_expert_offset,
                            int32_t inter_planes, const void* w13, const float* w13_scale, const void* w2,
                            const float* w2_scale, float* out_rows, void* workspace, size_t ws_bytes,
                            gemms_stream_t stream) {
  if (!info) return GEMMS_ERR_ARG;
  return ep_expert_ffn_impl(recv_buf, R_cap, info + kInfoR, P_max, H, I, top_k, E_local, local_expert_offset,
                            inter_planes, w13, w13_scale, w2, w2_scale, out_rows, workspace, ws_bytes, stream);
}

size_t gemms_ep_region_bytes(int32_t send_cap, int32_t H, int32_t top_k) {
  if (send_cap < 0 || H <= 0 || H % kBlock || top_k < 1 || top_k > 16) return 0;
  return kEpHdrBytes + (size_t)send_cap * ep_row_bytes(H, top_k);
}

int gemms_ep_pull(const void* const* region, int32_t rank, int32_t world, int32_t H, int32_t top_k,
                  int32_t send_cap, int32_t recv_cap, void* recv_buf, int32_t* info, gemms_stream_t stream_) {
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world || H <= 0 || H % kBlock || top_k < 1 ||
      top_k > 16 || send_cap < 0 || recv_cap < 0)
    return GEMMS_ERR_SHAPE;
  if (!region || !info || (!recv_buf && recv_cap > 0)) return GEMMS_ERR_ARG;
  if ((recv_buf && !aligned16(recv_buf)) || (reinterpret_cast<uintptr_t>(info) & 3u)) return GEMMS_ERR_ALIGN;
  PeerRegions reg{};
  for (int s = 0; s < world; ++s) {
    if (!region[s]) return GEMMS_ERR_ARG;
    if (!aligned16(region[s])) return GEMMS_ERR_ALIGN;
    reg.base[s] = static_cast<const uint8_t*>(region[s]);
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
  ep_pull_plan_kernel<<<1, 32, 0, st>>>(reg, rank, world, send_cap, recv_cap, info);
  GEMMS_CUDA_TRY(cudaGetLastError());
  if (recv_cap == 0) return GEMMS_OK;
  const int blocks = std::min(recv_cap, pull_ctas() > 0 ? pull_ctas() : num_sms() * 2);
  ep_pull_rows_kernel<<<blocks, 256, 0, st>>>(reg, info, world, ep_row_bytes(H, top_k),
                                               static_cast<uint8_t*>(recv_buf));
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}

int gemms_ep_pack_back_dev(const float* rows, int32_t R_cap, const int32_t* info, int32_t H, void* packed,
                           gemms_stream_t stream_) {
  if (R_cap < 0 || H <= 0 || H % 4) return GEMMS_ERR_SHAPE;
  if (R_cap == 0) return GEMMS_OK;
  if (!rows || !packed || !info) return GEMMS_ERR_ARG;
  if (!aligned16(rows) || !aligned16(packed)) return GEMMS_ERR_ALIGN;
  ep_pack_back_kernel<<<R_cap, 256, 0, reinterpret_cast<cudaStream_t>(stream_)>>>(
      rows, info + kInfoR, H, static_cast<uint8_t*>(packed), ep_back_row_bytes(H));
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}

int gemms_ep_combine_peer(const float* acc, const void* const* row_base, const int32_t* info,
                          const int32_t* send_row_of, int32_t T, int32_t H, int32_t world, int32_t recv_cap,
                          void* out_bf16, gemms_stream_t stream_) {
  if (T < 0 || H <= 0 || H % 4 || world < 1 || world > kMaxWorld || recv_cap < 1) return GEMMS_ERR_SHAPE;
  if (!acc || !send_row_of || !out_bf16 || !row_base || !info) return GEMMS_ERR_ARG;
  if (!aligned16(acc) || !aligned16(out_bf16)) return GEMMS_ERR_ALIGN;
  if (T == 0) return GEMMS_OK;
  BackRows at{};
  for (int d = 0; d < world; ++d) {
    if (row_base[d] && !aligned16(row_base[d])) return GEMMS_ERR_ALIGN;
    at.base[d] = static_cast<const uint8_t*>(row_base[d]);
  }
  at.add_dev = info + kInfoAdd;
  at.cap = recv_cap;
  ep_combine_kernel<<<T, 256, 0, reinterpret_cast<cudaStream_t>(stream_)>>>(
      acc, at, ep_back_row_bytes(H), send_row_of, T, H, world, static_cast<__nv_bfloat16*>(out_bf16), nullptr);
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}

int gemms_ep_gather_add_peer(float* acc, const void* const* row_base, const int32_t* info,
                             const int32_t* send_row_of, int32_t T, int32_t H, int32_t world, int32_t recv_cap,
                             gemms_stream_t stream_) {
  if (T < 0 || H <= 0 || H % 4 || world < 1 || world > kMaxWorld || recv_cap < 1) return GEMMS_ERR_SHAPE;
  if (!acc || !send_row_of || !row_base || !info) return GEMMS_ERR_ARG;
  if (!aligned16(acc)) return GEMMS_ERR_ALIGN;
  if (T == 0) return GEMMS_OK;
  BackRows at{};
  for (int d = 0; d < world; ++d) {
    if (row_base[d] && !aligned16(row_base[d])) return GEMMS_ERR_ALIGN;
    at.base[d] = static_cast<const uint8_t*>(row_base[d]);
  }
  at.add_dev = info + kInfoAdd;
  at.cap = recv_cap;
  ep_combine_kernel<<<T, 256, 0, reinterpret_cast<cudaStream_t>(stream_)>>>(
      nullptr, at, ep_back_row_bytes(H), send_row_of, T, H, world, nullptr, acc);
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}

int gemms_f32_to_bf16(const float* in, void* out_bf16, size_t n, gemms_stream_t stream) {
  if (n % 4) return GEMMS_ERR_SHAPE;
  if (n == 0) return GEMMS_OK;
  if (!in || !out_bf16) return GEMMS_ERR_ARG;
  if (!aligned16(in) || (reinterpret_cast<uintptr_t>(out_bf16) & 7u)) return GEMMS_ERR_ALIGN;
  return launch_to_bf16(in, static_cast<__nv_bfloat16*>(out_bf16), n, nullptr, reinterpret_cast<cudaStream_t>(stream));
}

int gemms_ep_set_pull_ctas(int32_t ctas) {
  if (ctas < 0) return GEMMS_ERR_ARG;
  return g_pull_ctas.exchange(ctas);
}

size_t gemms_ep_back_row_bytes(int32_t H) { return H > 0 ? ep_back_row_bytes(H) : 0; }

int gemms_ep_pack_back(const float* rows, int32_t R, int32_t H, void* packed, gemms_stream_t stream_) {
  if (R < 0 || H <= 0 || H % 4) return GEMMS_ERR_SHAPE;
  if (R == 0) return GEMMS_OK;
  if (!rows || !packed) return GEMMS_ERR_ARG;
  if (!aligned16(rows) || !aligned16(packed)) return GEMMS_ERR_ALIGN;
  ep_pack_back_kernel<<<R, 256, 0, reinterpret_cast<cudaStream_t>(stream_)>>>(
      rows, nullptr, H, static_cast<uint8_t*>(packed), ep_back_row_bytes(H));
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}

int gemms_ep_combine(const float* acc, const void* back_packed, const int32_t* send_row_of, int32_t T, int32_t H,
                     int32_t world, void* out_bf16, gemms_stream_t stream_) {
  if (T < 0 || H <= 0 || H % 4 || world < 1 || world > kMaxWorld) return GEMMS_ERR_SHAPE;
  if (!acc || !send_row_of || !out_bf16) return GEMMS_ERR_ARG;  // back_packed may be NULL when nothing was sent
  if (!aligned16(acc) || !aligned16(out_bf16) || (back_packed && !aligned16(back_packed))) return GEMMS_ERR_ALIGN;
  if (T == 0) return GEMMS_OK;
  BackRows at{};
  for (int d = 0; d < world; ++d) at.base[d] = static_cast<const uint8_t*>(back_packed);
  ep_combine_kernel<<<T, 256, 0, reinterpret_cast<cudaStream_t>(stream_)>>>(
      acc, at, ep_back_row_bytes(H), send_row_of, T, H, world, static_cast<__nv_bfloat16*>(out_bf16), nullptr);
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}

int gemms_ep_combine_rows(const float* acc, const void* const* row_base, const int32_t* row_add,
                          const int32_t* send_row_of, int32_t T, int32_t H, int32_t world, void* out_bf16,
                          gemms_stream_t stream_) {
  if (T < 0 || H <= 0 || H % 4 || world < 1 || world > kMaxWorld) return GEMMS_ERR_SHAPE;
  if (!acc || !send_row_of || !out_bf16 || !row_base || !row_add) return GEMMS_ERR_ARG;
  if (!aligned16(acc) || !aligned16(out_bf16)) return GEMMS_ERR_ALIGN;
  if (T == 0) return GEMMS_OK;
  BackRows at{};
  for (int d = 0; d < world; ++d) {
    if (row_base[d] && !aligned16(row_base[d])) return GEMMS_ERR_ALIGN;
    at.base[d] = static_cast<const uint8_t*>(row_base[d]);
    at.add[d] = row_add[d];
  }
  ep_combine_kernel<<<T, 256, 0, reinterpret_cast<cudaStream_t>(stream_)>>>(
      acc, at, ep_back_row_bytes(H), send_row_of, T, H, world, static_cast<__nv_bfloat16*>(out_bf16), nullptr);
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}

}  // extern "C"
