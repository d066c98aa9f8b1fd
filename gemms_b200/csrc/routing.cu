// routing.cu -- DeepSeek-V3 no-aux grouped router, M-tile planning and
// deterministic expert-grouped row assignment.
//
// Reference: routing in flashinfer_baseline.py:95-127 (the oracle);
// routing_topk_kernel persistent_kernel2.cu:153-299 and
// routing_permute_kernel persistent_kernel2.cu:308-346 (the reference's GPU
// attempt, which hard-codes group size 32, uses ex2.approx for the sigmoid
// and assigns rows with atomics, i.e. in nondeterministic order).
#include "common.cuh"
#include <algorithm>
#include <cfloat>

namespace gemms {
namespace {

constexpr int kMaxV = 8;  // experts per lane: E <= 256

struct Top2 {
  float a, b;  // a >= b
};

__device__ __forceinline__ Top2 merge_top2(Top2 x, Top2 y) {
  Top2 r;
  r.a = fmaxf(x.a, y.a);
  r.b = fmaxf(fminf(x.a, y.a), fmaxf(x.b, y.b));
  return r;
}

// (value, index) arg-max with ties broken towards the smaller index.
__device__ __forceinline__ void argmax_merge(float& v, int& i, float ov, int oi) {
  if (ov > v || (ov == v && oi < i)) {
    v = ov;
    i = oi;
  }
}

// pp[0] + pp[stride] + ... + pp[(n-1)*stride], added in index order; the loads
// are issued eight at a time (independent), only the additions are chained.
__device__ __forceinline__ float sum_partials_in_order(const float* pp, int n, size_t stride) {
  float x = 0.f;
  for (int q0 = 0; q0 < n; q0 += 8) {
    float v[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) v[q] = q0 + q < n ? pp[(size_t)(q0 + q) * stride] : 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q)
      if (q0 + q < n) x = (q0 + q == 0) ? v[q] : __fadd_rn(x, v[q]);
  }
  return x;
}

// Order-preserving map of fp32 to uint32 (larger float -> larger key) for the
// warp-wide integer max/min reductions.  The router never compares -0.0 (a
// sum with a positive sigmoid is never -0), so equal keys are equal floats.
__device__ __forceinline__ uint32_t f2key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// One warp per token.  Lane l holds experts e = j*32 + l (j < V).
// Sigmoid: exp is evaluated in double and rounded to fp32 (correctly rounded
// in practice), then 1/(1+e) and + bias in IEEE fp32 -- the oracle computes
// the same values (oracle/reference_moe.py: sigmoid_exact).
__global__ void __launch_bounds__(256) route_kernel(RouteArgs a) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= a.T) return;
  const int E = a.E;
  const int V = (E + 31) >> 5;
  const int gs = E / a.n_group;  // power of two in [2, 32]

  float s[kMaxV], sb[kMaxV];
#pragma unroll
  for (int j = 0; j < kMaxV; ++j) {
    s[j] = 0.f;
    sb[j] = -INFINITY;
    const int e = j * 32 + lane;
    if (j < V && e < E) {
      float x;
      if (a.partials) {
        // router-GEMM split-K partials, summed in split order (deterministic)
        x = sum_partials_in_order(a.partials + (size_t)t * E + e, a.n_partials, (size_t)a.T * E);
        if (a.logits_out) a.logits_out[(size_t)t * E + e] = x;
      } else {
        x = __ldg(a.logits + (size_t)t * E + e);
      }
      const float ex = static_cast<float>(exp(-static_cast<double>(x)));
      s[j] = __fdiv_rn(1.0f, __fadd_rn(1.0f, ex));
      const float bias = a.bias_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.bias)[e])
                                     : reinterpret_cast<const float*>(a.bias)[e];
      sb[j] = __fadd_rn(s[j], bias);
    }
  }

  // Group score = sum of the two largest biased scores of the group
  // (flashinfer_baseline.py:108-109).  Groups are aligned lane segments of
  // width gs within one register j.
  bool kept[kMaxV];
#pragma unroll
  for (int j = 0; j < kMaxV; ++j) kept[j] = false;
  if (gs == 32) {
    float gscore[kMaxV];
    // One group per register (DeepSeek-V3: 8 groups of 32): the group's
    // largest key by one warp max, the second by another unless the largest
    // occurs twice; the group scores are then the same in every lane, and
    // every lane picks the kept groups in registers, by (score desc, group
    // asc) as below.
#pragma unroll
    for (int j = 0; j < kMaxV; ++j) {
      gscore[j] = -INFINITY;
      if (j < V) {
        const uint32_t k = f2key(sb[j]);
        const uint32_t m1 = __reduce_max_sync(0xffffffffu, k);
        uint32_t m2 = m1;
        if (__popc(__ballot_sync(0xffffffffu, k == m1)) < 2) m2 = __reduce_max_sync(0xffffffffu, k == m1 ? 0u : k);
        gscore[j] = __fadd_rn(key2f(m1), key2f(m2));
      }
    }
    for (int it = 0; it < a.topk_group; ++it) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < kMaxV; ++j)
        if (j < V && !kept[j]) argmax_merge(bv, bi, gscore[j], j);
#pragma unroll
      for (int j = 0; j < kMaxV; ++j)
        if (j == bi) kept[j] = true;
    }
  } else {
  float gscore[kMaxV];
#pragma unroll
  for (int j = 0; j < kMaxV; ++j) {
    Top2 t2{sb[j], -INFINITY};
    for (int off = 1; off < gs; off <<= 1) {
      Top2 o{__shfl_xor_sync(0xffffffffu, t2.a, off), __shfl_xor_sync(0xffffffffu, t2.b, off)};
      t2 = merge_top2(t2, o);
    }
    gscore[j] = __fadd_rn(t2.a, t2.b);
  }

  // Keep the topk_group best groups (:112-115).  Group id of (j, lane) is
  // (j*32 + lane) / gs; one lane per group segment proposes its score.
  for (int it = 0; it < a.topk_group; ++it) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < kMaxV; ++j) {
      const int e = j * 32 + lane;
      if (j < V && e < E && (lane % gs) == 0 && !kept[j]) argmax_merge(bv, bi, gscore[j], e / gs);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      argmax_merge(bv, bi, ov, oi);
    }
#pragma unroll
    for (int j = 0; j < kMaxV; ++j) {
      const int e = j * 32 + lane;
      if (j < V && e < E && e / gs == bi) kept[j] = true;
    }
  }
  }

  // Top-k over biased scores of experts in kept groups (:118-120).
  float cand[kMaxV];
#pragma unroll
  for (int j = 0; j < kMaxV; ++j) cand[j] = kept[j] ? sb[j] : -INFINITY;
  int my_e = -1;
  float my_s = 0.f;
  for (int it = 0; it < a.top_k; ++it) {
    float bv = -INFINITY, bs = 0.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < kMaxV; ++j) {
      const int e = j * 32 + lane;
      if (cand[j] > bv || (cand[j] == bv && cand[j] > -INFINITY && e < bi)) {
        bv = cand[j];
        bi = e;
        bs = s[j];
      }
    }
    // warp-wide best (value desc, index asc): the largest key, then the
    // smallest index among the lanes holding it.  The winner is its owner
    // lane's own best, so that lane's bs is its unbiased score (0 once no
    // candidate is left).
    const uint32_t kb = f2key(bv);
    const uint32_t mk = __reduce_max_sync(0xffffffffu, kb);
    bi = static_cast<int>(__reduce_min_sync(0xffffffffu, kb == mk ? static_cast<uint32_t>(bi) : 0x7fffffffu));
    const float bs_owner = __shfl_sync(0xffffffffu, bs, bi & 31);
    bs = bi == 0x7fffffff ? 0.f : bs_owner;
    if (lane == it) {
      my_e = bi;
      my_s = bs;
    }
#pragma unroll
    for (int j = 0; j < kMaxV; ++j)
      if (j * 32 + lane == bi) cand[j] = -INFINITY;
  }

  // weights = s / (sum of selected s + 1e-20) * rsf  (:123-127)
  float sum = (lane < a.top_k) ? my_s : 0.f;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  sum = __fadd_rn(sum, 1e-20f);
  if (lane < a.top_k) {
    const size_t o = (size_t)t * a.top_k + lane;
    a.topk_idx[o] = my_e;
    a.topk_w[o] = __fmul_rn(__fdiv_rn(my_s, sum), a.rsf);
    if (a.pair_row) a.pair_row[o] = -1;
    const int le = my_e - a.local_offset;
    if (a.counts && le >= 0 && le < a.E_local) atomicAdd(a.counts + le, 1);
  }
}

// Decode-sized batches: one 256-thread block per token, thread e owns expert e
// (E <= 256), so the token's dependency chain (group scores, group choice,
// top-k) is spread over 8 warps instead of running in one.  Same arithmetic
// as route_kernel and the same (value desc, index asc) order at every choice,
// so the results are identical: each warp keeps its own top-k of the kept
// candidates, and warp 0 picks the global top-k from those lists (the global
// top-k under a strict order lies in the union of the warps' top-k).
constexpr int kRouteBlockMaxT = 64;

struct RouteBlockSmem {
  float g[256];  // group scores (n_group <= E / 2)
  int kept[256];
  float v[8][16], s[8][16];
  int i[8][16];
};

// The routing of token t by 256 threads (tid = 0..255 within the group).  All
// threads of the block call it the same number of times: it has three block
// barriers; a group whose token is past T (active false) only joins them.
__device__ __forceinline__ void route_block_body(const RouteArgs& a, int t, bool active, int tid,
                                                 RouteBlockSmem& sm, int32_t* s_counts) {
  float* s_g = sm.g;
  int* s_kept = sm.kept;
  auto& s_v = sm.v;
  auto& s_s = sm.s;
  auto& s_i = sm.i;
  const unsigned full = 0xffffffffu;
  const int lane = tid & 31, warp = tid >> 5;
  const int E = a.E, ng = a.n_group;
  const int gs = E / ng;
  const int e = tid;
  const bool live = active && e < E;
  float s = 0.f, sb = -INFINITY;
  if (live) {
    float x;
    if (a.partials) {
      x = sum_partials_in_order(a.partials + (size_t)t * E + e, a.n_partials, (size_t)a.T * E);
      if (a.logits_out) a.logits_out[(size_t)t * E + e] = x;
    } else {
      x = __ldg(a.logits + (size_t)t * E + e);
    }
    const float ex = static_cast<float>(exp(-static_cast<double>(x)));
    s = __fdiv_rn(1.0f, __fadd_rn(1.0f, ex));
    const float bias = a.bias_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.bias)[e])
                                   : reinterpret_cast<const float*>(a.bias)[e];
    sb = __fadd_rn(s, bias);
  }
  // group score: sum of the group's two largest biased scores (segmented butterfly)
  Top2 t2{sb, -INFINITY};
  for (int off = 1; off < gs; off <<= 1) {
    Top2 o{__shfl_xor_sync(full, t2.a, off), __shfl_xor_sync(full, t2.b, off)};
    t2 = merge_top2(t2, o);
  }
  if (live && e % gs == 0) s_g[e / gs] = __fadd_rn(t2.a, t2.b);
  __syncthreads();
  if (active && warp == 0) {  // the topk_group best groups
    for (int g = lane; g < ng; g += 32) s_kept[g] = 0;
    __syncwarp();
    for (int it = 0; it < a.topk_group; ++it) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int g = lane; g < ng; g += 32)
        if (!s_kept[g]) argmax_merge(bv, bi, s_g[g], g);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(full, bv, off);
        const int oi = __shfl_xor_sync(full, bi, off);
        argmax_merge(bv, bi, ov, oi);
      }
      if (lane == 0 && bi >= 0 && bi < ng) s_kept[bi] = 1;
      __syncwarp();
    }
  }
  __syncthreads();
  // each warp: its 32 candidates sorted best first by (biased score desc,
  // expert index asc) with a bitonic network; lanes < top_k hold its top-k.
  // Non-candidates carry (-inf, 0x7fffffff, 0), the value route_kernel's
  // selection reports once no candidate is left.
  float v = (live && s_kept[e / gs]) ? sb : -INFINITY;
  int vi = v > -INFINITY ? e : 0x7fffffff;
  float vs = v > -INFINITY ? s : 0.f;
  auto better = [](float v1, int i1, float v2, int i2) { return v1 > v2 || (v1 == v2 && i1 < i2); };
#pragma unroll
  for (int kk = 2; kk <= 32; kk <<= 1) {
#pragma unroll
    for (int j = kk >> 1; j > 0; j >>= 1) {
      const float ov = __shfl_xor_sync(full, v, j);
      const int oi = __shfl_xor_sync(full, vi, j);
      const float os = __shfl_xor_sync(full, vs, j);
      const bool lower = (lane & j) == 0, best_first = (lane & kk) == 0;
      const bool take = (lower == best_first) ? better(ov, oi, v, vi) : better(v, vi, ov, oi);
      if (take) {
        v = ov;
        vi = oi;
        vs = os;
      }
    }
  }
  if (lane < a.top_k) {
    s_v[warp][lane] = v;
    s_i[warp][lane] = vi;
    s_s[warp][lane] = vs;
  }
  __syncthreads();
  if (!active || warp != 0) return;
  // warp 0: merge the 8 sorted lists, lane w < 8 holding list w's head
  int head = 0;
  int my_e = -1;
  float my_s = 0.f;
  for (int it = 0; it < a.top_k; ++it) {
    const bool has = lane < 8 && head < a.top_k;
    float bv = has ? s_v[lane & 7][head] : -INFINITY;
    int bi = has ? s_i[lane & 7][head] : 0x7fffffff;
    float bs = has ? s_s[lane & 7][head] : 0.f;
    const float pv = bv;
    const int pi = bi;
#pragma unroll
    for (int off = 4; off > 0; off >>= 1) {  // within lanes 0-7 (and within each later group of 8)
      const float ov = __shfl_xor_sync(full, bv, off);
      const int oi = __shfl_xor_sync(full, bi, off);
      const float os = __shfl_xor_sync(full, bs, off);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
        bs = os;
      }
    }
    bv = __shfl_sync(full, bv, 0);
    bi = __shfl_sync(full, bi, 0);
    bs = __shfl_sync(full, bs, 0);
    if (lane == it) {
      my_e = bi;
      my_s = bs;
    }
    // the list that supplied the winner moves on (lowest such lane for fillers)
    const unsigned hit = __ballot_sync(full, lane < 8 && pv == bv && pi == bi);
    if (hit && lane == __ffs(hit) - 1) ++head;
  }
  float sum = (lane < a.top_k) ? my_s : 0.f;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(full, sum, off);
  sum = __fadd_rn(sum, 1e-20f);
  if (lane < a.top_k) {
    const size_t o = (size_t)t * a.top_k + lane;
    a.topk_idx[o] = my_e;
    a.topk_w[o] = __fmul_rn(__fdiv_rn(my_s, sum), a.rsf);
    if (a.pair_row) a.pair_row[o] = -1;
    const int le = my_e - a.local_offset;
    if (le >= 0 && le < a.E_local) {
      if (s_counts) atomicAdd(s_counts + le, 1);
      else if (a.counts) atomicAdd(a.counts + le, 1);
    }
  }
}

__global__ void __launch_bounds__(256) route_block_kernel(RouteArgs a) {
  __shared__ RouteBlockSmem sm;
  route_block_body(a, blockIdx.x, true, threadIdx.x, sm, nullptr);
}

// Single block: per-group exclusive offsets and the 128-row M-tile list.
// Needs blockDim.x == 1024 (the scan width); every thread of the block calls it.
__device__ __forceinline__ void plan_block(const PlanArgs& a, int* s_tiles, int* s_rows) {
  const int groups = a.E_local + (a.shared_rows > 0 ? 1 : 0);
  const int tid = threadIdx.x;
  int rows_total = 0, tiles_total = 0;
  // Chunked scan over groups (groups may exceed blockDim in principle).
  for (int base = 0; base < groups; base += blockDim.x) {
    const int g = base + tid;
    int c = 0;
    if (g < groups) c = (g < a.E_local) ? a.counts[g] : a.shared_rows;
    s_rows[tid] = c;
    s_tiles[tid] = (c + kBlock - 1) / kBlock;
    __syncthreads();
    for (int off = 1; off < (int)blockDim.x; off <<= 1) {
      int vr = 0, vt = 0;
      if (tid >= off) {
        vr = s_rows[tid - off];
        vt = s_tiles[tid - off];
      }
      __syncthreads();
      s_rows[tid] += vr;
      s_tiles[tid] += vt;
      __syncthreads();
    }
    const int incl_r = s_rows[tid], incl_t = s_tiles[tid];
    const int row0 = rows_total + incl_r - c;
    const int tile0 = tiles_total + incl_t - (c + kBlock - 1) / kBlock;
    if (g < groups) {
      a.offsets[g] = row0;
      if (a.group_tile0) a.group_tile0[g] = tile0;
      const int nt = (c + kBlock - 1) / kBlock;
      for (int i = 0; i < nt; ++i) {
        const int ti = tile0 + i;
        if (ti < a.max_tiles) {
          a.tile_group[ti] = g;
          a.tile_row0[ti] = row0 + i * kBlock;
          a.tile_rows[ti] = min(kBlock, c - i * kBlock);
        } else {
          atomicOr(a.err, kErrRowOverflow);
        }
      }
    }
    rows_total += s_rows[blockDim.x - 1];
    tiles_total += s_tiles[blockDim.x - 1];
    __syncthreads();
  }
  if (tid == 0) {
    a.offsets[groups] = rows_total;
    if (a.group_tile0) a.group_tile0[groups] = tiles_total;
    a.num_tiles[0] = min(tiles_total, a.max_tiles);
    if (rows_total > a.row_capacity) {  // counts disagree with the buffers' size: do no GEMM work
      a.num_tiles[0] = 0;
      atomicOr(a.err, kErrRowOverflow);
    }
  }
}

__global__ void __launch_bounds__(1024) plan_kernel(PlanArgs a) {
  __shared__ int s_tiles[1024];
  __shared__ int s_rows[1024];
  plan_block(a, s_tiles, s_rows);
}

// Decode-sized batches (T <= kFrontMaxT): routing, plan and row assignment
// in one 1024-thread block, four groups of 256 threads routing one token each
// (route_block_body), then plan_block over the block's counts, then the rows
// of each local expert in increasing token order.  The results are those of
// route_block_kernel + plan_kernel + assign_kernel; the two launches and
// kernel boundaries it saves are a large part of a decode step.
constexpr int kFrontMaxT = 4;

__global__ void __launch_bounds__(1024) decode_front_kernel(RouteArgs ra, PlanArgs pa, AssignArgs sa,
                                                           float* __restrict__ zero_buf, size_t zero_n) {
  __shared__ RouteBlockSmem rsm[kFrontMaxT];
  __shared__ int32_t s_counts[256];
  __shared__ int s_tiles[1024];
  __shared__ int s_rows[1024];
  const int tid = threadIdx.x;
  if (tid < 256) s_counts[tid] = 0;
  for (size_t i = tid; zero_buf && i < zero_n; i += blockDim.x) zero_buf[i] = 0.f;  // the layer's fp32 accumulator
  __syncthreads();
  const int t = tid >> 8;  // this thread's token group
  route_block_body(ra, t, t < ra.T, tid & 255, rsm[t], s_counts);
  __syncthreads();
  for (int i = tid; i < ra.E_local; i += blockDim.x) ra.counts[i] = s_counts[i];
  __syncthreads();
  plan_block(pa, s_tiles, s_rows);
  __syncthreads();
  const int K = sa.top_k;
  if (tid < sa.T * K) {  // (token, slot): its rank among the tokens routed to the same expert
    const int tt = tid / K, j = tid - tt * K;
    const int e = sa.topk_idx[tt * K + j];
    const int le = e - sa.local_offset;
    if (e >= 0 && le >= 0 && le < sa.E_local) {
      int rank = 0;
      for (int tp = 0; tp < tt; ++tp)
        for (int jp = 0; jp < K; ++jp) rank += sa.topk_idx[tp * K + jp] == e;
      const int r = sa.offsets[le] + rank;
      if (r < sa.row_capacity) {
        sa.row_token[r] = tt;
        sa.row_weight[r] = sa.topk_w[tt * K + j];
        sa.pair_row[tt * K + j] = r;
      }
    }
  }
  if (sa.shared_rows > 0 && tid < sa.T) {
    const int r = sa.offsets[sa.E_local] + tid;
    if (r < sa.row_capacity) {
      sa.row_token[r] = tid;
      sa.row_weight[r] = 1.0f;
    }
  }
}

// One block per local expert: rows are assigned in increasing token order,
// so the grouped layout is deterministic (unlike atomics-based permutes).
__global__ void __launch_bounds__(1024) assign_kernel(AssignArgs a) {
  __shared__ int s_warp[32];
  __shared__ int s_base;
  const int le = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  const int T = a.T_dev ? min(a.T, *a.T_dev) : a.T;
  if (le == a.E_local) {  // shared expert group: row offsets[E_local] + t
    const int r0 = a.offsets[a.E_local];
    for (int t = tid; t < T && r0 + t < a.row_capacity; t += blockDim.x) {
      a.row_token[r0 + t] = t;
      a.row_weight[r0 + t] = 1.0f;
    }
    return;
  }
  const int ge = a.local_offset + le;
  const int stride = a.idx_stride > 0 ? a.idx_stride : a.top_k;
  if (tid == 0) s_base = a.offsets[le];
  __syncthreads();
  for (int t0 = 0; t0 < T; t0 += blockDim.x) {
    const int t = t0 + tid;
    int jsel = -1;
    if (t < T) {
      for (int j = 0; j < a.top_k; ++j)
        if (a.topk_idx[(size_t)t * stride + j] == ge) jsel = j;
    }
    const unsigned ballot = __ballot_sync(0xffffffffu, jsel >= 0);
    if (lane == 0) s_warp[warp] = __popc(ballot);
    __syncthreads();
    if (warp == 0) {
      int v = lane < nwarps ? s_warp[lane] : 0;
      for (int off = 1; off < 32; off <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, v, off);
        if (lane >= off) v += o;
      }
      if (lane < nwarps) s_warp[lane] = v;  // inclusive
    }
    __syncthreads();
    const int warp_excl = (warp > 0 ? s_warp[warp - 1] : 0);
    const int base = s_base;
    const int r = base + warp_excl + __popc(ballot & ((1u << lane) - 1u));
    if (jsel >= 0 && r < a.row_capacity) {
      a.row_token[r] = t;
      a.row_weight[r] = a.topk_w[(size_t)t * stride + jsel];
      a.pair_row[(size_t)t * a.top_k + jsel] = r;
    }
    __syncthreads();
    if (tid == 0) s_base = base + s_warp[nwarps - 1];
    __syncthreads();
  }
}

// logits[t][e] = sum over q of partials[q][t][e], in split order (as route_kernel).
__global__ void sum_partials_kernel(const float* __restrict__ partials, int splits, size_t n, float* __restrict__ out) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    float x = partials[i];
    for (int q = 1; q < splits; ++q) x = __fadd_rn(x, partials[(size_t)q * n + i]);
    out[i] = x;
  }
}

}  // namespace

int launch_sum_partials(const float* partials, int splits, int T, int E, float* logits, cudaStream_t s) {
  const size_t n = (size_t)T * E;
  if (n == 0) return GEMMS_OK;
  const int blocks = static_cast<int>(std::min<size_t>((n + 255) / 256, (size_t)num_sms() * 8));
  sum_partials_kernel<<<blocks, 256, 0, s>>>(partials, splits, n, logits);
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}

int launch_route(const RouteArgs& a, cudaStream_t s) {
  if (a.T <= 0) return GEMMS_OK;
  if (a.T <= kRouteBlockMaxT && a.E <= 256 && a.top_k <= 16) {
    route_block_kernel<<<a.T, 256, 0, s>>>(a);
    GEMMS_CUDA_TRY(cudaGetLastError());
    return GEMMS_OK;
  }
  const int warps_per_block = 8;
  route_kernel<<<cdiv(a.T, warps_per_block), warps_per_block * 32, 0, s>>>(a);
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}

bool decode_front_ok(const RouteArgs& ra, const PlanArgs& pa) {
  return ra.T >= 1 && ra.T <= kFrontMaxT && ra.E <= 256 && ra.top_k <= 16 && ra.E_local <= 256 &&
         pa.E_local + (pa.shared_rows > 0 ? 1 : 0) <= 1024;
}

int launch_decode_front(const RouteArgs& ra, const PlanArgs& pa, const AssignArgs& sa, float* zero_buf, size_t zero_n,
                        cudaStream_t s) {
  if (!decode_front_ok(ra, pa) || sa.idx_stride > 0 || sa.T_dev) return GEMMS_ERR_SHAPE;
  decode_front_kernel<<<1, 1024, 0, s>>>(ra, pa, sa, zero_buf, zero_n);
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}

int launch_plan(const PlanArgs& a, cudaStream_t s) {
  plan_kernel<<<1, 1024, 0, s>>>(a);
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}

int launch_assign(const AssignArgs& a, cudaStream_t s) {
  const int blocks = a.E_local + (a.shared_rows > 0 ? 1 : 0);
  if (blocks == 0 || a.T <= 0) return GEMMS_OK;
  // few tokens: a block as wide as the tokens (whole warps), not 1024 idle threads
  const int threads = a.T_dev ? 1024 : std::min(1024, std::max(32, (a.T + 31) / 32 * 32));
  assign_kernel<<<blocks, threads, 0, s>>>(a);
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}

}  // namespace gemms
