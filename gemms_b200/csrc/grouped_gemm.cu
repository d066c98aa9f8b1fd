// grouped_gemm.cu -- grouped, 128x128 block-scaled FP8 GEMMs on tcgen05.
//
// GEMM1 (gate/up projection + SwiGLU) and GEMM2 (down projection + routing
// weight + combine) of the MoE layer.  Reference: the per-expert loop of the
// oracle, flashinfer_baseline.py:135-167 (G1 = A_e W13_e^T; C = silu(G1[:,I:])
// * G1[:,:I]; O = C W2_e^T; out += w * O), and the reference's attempt at it,
// persistent_gemm_kernel in persistent_kernel2.cu:388-890.
//
// Design (one persistent CTA per SM, 384 threads, warp-specialised; the
// control warpgroup 0-3 runs on 40-56 registers, the epilogue warpgroups on
// 224-232 via setmaxnreg):
//   warp 0      TMA producer: A tile(s) [128 rows x 128 B] per plane and two
//               128-row weight boxes per stage into a 2-4 deep smem ring.
//   warp 1      allocates all 512 TMEM columns and issues tcgen05.mma
//               (M=128, N=256, K=32 e4m3) from one thread; each 128-wide K
//               block goes to one of two TMEM partial accumulators.
//   warps 2-3   idle (setmaxnreg works per warpgroup).
//   warps 4-11  "promotion" epilogue: for every K block read the fp32 partial
//               from TMEM, multiply by a_scale[row,kb] * w_scale[nblk,kb] and
//               accumulate in registers (the block scales are arbitrary fp32,
//               so the MX block-scaled MMA kinds cannot absorb them).  Then:
//               GEMM1: SwiGLU, then re-quantise C per 1x128 into PLANES e4m3
//                      planes sharing one scale (hi, residual, ...), so GEMM2
//                      sums the planes in the same TMEM accumulator.
//               GEMM2: scale by the routing weight and add the fp32 row into
//                      the token's output row with vector atomics.
// Work units are (M tile, N tile) with N fastest: CTAs working on adjacent
// units share the A tile, and the M tiles of one expert are adjacent so their
// weight tiles are read from HBM once and from L2 after that.
#include "common.cuh"
#include "sm100.cuh"

#include <atomic>
#include <cudaTypedefs.h>
#include <cstdlib>
#include <cstring>
#include <mutex>

namespace gemms {
namespace {
using namespace sm100;

constexpr int BM = 128;                 // rows per tile = TMEM lanes
constexpr int BN = 256;                 // output columns per tile
constexpr int BK = 128;                 // K (bytes) per stage = one scale block
constexpr int UMMA_K = 32;              // K per tcgen05.mma for 8-bit inputs
constexpr int kThreads = 384;          // 3 warpgroups
constexpr int kEpiWarps = 8;           // warpgroups 1-2
constexpr int kEpiFirstWarp = 4;
// Register split (setmaxnreg): launched at 168/thread (384 threads), the
// producer/MMA warpgroup drops to `ctrl` and the two epilogue warpgroups rise
// to `epi`, with ctrl + 2 x epi <= 504 <= 512 registers per lane of an SM
// sub-partition and 4x32xctrl + 8x32xepi <= 64512 = 384 x 168 (the launch
// allocation).  The epilogue share holds the 128 running sums plus two
// 32-column TMEM loads per wait without spilling.
// GEMM1's epilogue (SwiGLU + requant) needs the larger share; GEMM2's
// producer needs more than 40.  Both splits satisfy the budgets above.
template <int MODE> struct Regs {
  static constexpr int ctrl = MODE == 0 ? 40 : 56;
  static constexpr int epi = MODE == 0 ? 232 : 224;
};
constexpr uint32_t kTmemCols = 512;     // 2 partial accumulators x 256 columns
constexpr int kTileA = BM * BK;         // 16 KB
constexpr int kTileB = BN * BK;         // 32 KB

constexpr int kEpiWarpsCfg = 8;

template <int PLANES>
struct Cfg {
  static constexpr int kStageBytes = PLANES * kTileA + kTileB;
  static constexpr int kStages = PLANES == 1 ? 4 : (PLANES == 2 ? 3 : 2);
  static constexpr int kRingBytes = kStages * kStageBytes;
  // GEMM2 (PLANES > 1) stages its combine writes: 8 warps x 32 rows x 20 floats.
  static constexpr int kStageOutBytes = PLANES > 1 ? kEpiWarpsCfg * 32 * 20 * 4 : 0;
  static constexpr int kSmemBytes = kRingBytes + 4096 + kStageOutBytes + 1024;  // + barriers/exchange + slack
};

struct GemmParams {
  const int32_t* tile_group;
  const int32_t* tile_row0;
  const int32_t* tile_rows;
  const int32_t* num_tiles;
  const int32_t* group_tile0;  // set: units ordered expert by expert, M tiles fastest (see unit_tile)
  int max_tiles;
  int shared_group;
  int n_tiles;       // N tiles per M tile
  int kb_count;      // K blocks
  int plane_stride;  // bytes between A planes within a row
  int w_rows;        // weight rows per expert
  int b_row_step;    // weight rows per N tile step
  int b_row_hi;      // row offset of the second 128-row weight box
  int prefetch;      // weight K-blocks prefetched into L2 ahead of the smem ring
  const float* a_scale;
  int a_scale_ld;
  const float* w_scale;   // [E, w_rows/128, kb_count]
  const float* sw_scale;  // [w_rows/128, kb_count]
  // GEMM1 epilogue
  uint8_t* inter;
  float* inter_scale;
  int inter_scale_ld;
  int I;
  // GEMM2 epilogue
  const int32_t* row_dest;
  const float* row_weight;
  float* out;
  float* pair_out;  // deterministic combine: weighted rows stored per grouped row, no atomics
  int H;
  int* err;
  // Bounded waits: cycles before a pipeline wait gives up (product default
  // GEMMS_WAIT_TIMEOUT_CYCLES).  stall_iter >= 0 is a test hook: CTA 0's
  // producer stops issuing at that K iteration (nothing left in flight), so
  // the MMA thread's wait for the missing stage runs out and reports
  // kErrGemmMmaWait through the error word.
  long long wait_limit;
  int stall_iter;
};

// Unit u -> (M tile, N tile).  Default: N fastest (consecutive CTAs share an A
// tile).  With group_tile0: within an expert, its M tiles are fastest, so the
// CTAs that read the same weight tile (one per M tile of the expert) run side
// by side and the second read finds the tile in L2.  The units of group g are
// [first_tile(g), first_tile(g + 1)) x n_tiles in either order.
__device__ __forceinline__ void unit_tile(const GemmParams& p, int u, int num_tiles, int& mt, int& nt) {
  const int mt0 = u / p.n_tiles;
  if (!p.group_tile0) {
    mt = mt0;
    nt = u - mt0 * p.n_tiles;
    return;
  }
  const int g = p.tile_group[mt0];
  const int t0 = p.group_tile0[g];
  const int c = min(p.group_tile0[g + 1], num_tiles) - t0;  // tiles of g that are listed
  const int v = u - t0 * p.n_tiles;
  mt = t0 + v % c;
  nt = v / c;
}

__device__ __forceinline__ uint16_t f2_to_e4m3x2(float a, float b) {
  return static_cast<uint16_t>(__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3));
}
__device__ __forceinline__ float2 e4m3x2_to_f2(uint16_t v) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(v), __NV_E4M3);
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

// Drain wait used on exit: bounded, ignores the abort flag, reports nothing.
__device__ __forceinline__ void mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() - t0 > GEMMS_WAIT_TIMEOUT_NS) return;
}

template <int MODE, int PLANES, int OUT_PLANES>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmBs, const GemmParams p) {
  using C = Cfg<PLANES>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kRingBytes);
  uint64_t* empty = full + S;
  uint64_t* pfull = empty + S;
  uint64_t* pempty = pfull + 2;
  uint64_t* mma_done = pempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* amax_x = reinterpret_cast<float*>(smem + C::kRingBytes + 512);  // [2 units][2 halves][128]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&pfull[b], 1);
      mbar_init(&pempty[b], kEpiWarps);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmBs);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // The TMEM base address is re-read from shared memory inside each role:
  // a value kept live across the role split was spilled to local memory and
  // reloaded once per K block by every epilogue warp and the MMA thread.

  const int num_tiles = min(*p.num_tiles, p.max_tiles);
  const int total = num_tiles * p.n_tiles;

  if (warp < kEpiFirstWarp) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(Regs<MODE>::ctrl));
   if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_a = policy_evict_last();
      // Weight coordinates of this CTA's it-th K iteration (units are strided
      // by gridDim.x); used both to load and to prefetch ahead into L2.
      const int my_units = total > (int)blockIdx.x ? (total - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
      const int my_iters = my_units * p.kb_count;
      auto weight_rows = [&](int it, int& kb, int& wrow, const CUtensorMap*& mb) {
        const int i = it / p.kb_count;
        kb = it - i * p.kb_count;
        const int u = blockIdx.x + i * gridDim.x;
        int mt, nt;
        unit_tile(p, u, num_tiles, mt, nt);
        const int g = p.tile_group[mt];
        const bool sh = (g == p.shared_group);
        mb = sh ? &tmBs : &tmB;
        wrow = (sh ? 0 : g * p.w_rows) + nt * p.b_row_step;
      };
      for (int pf = 0; pf < p.prefetch && pf < my_iters; ++pf) {
        int kb, wrow;
        const CUtensorMap* mb;
        weight_rows(pf, kb, wrow, mb);
        tma_prefetch_l2_2d(mb, kb * BK, wrow, pol_w);
        tma_prefetch_l2_2d(mb, kb * BK, wrow + p.b_row_hi, pol_w);
      }
      int it = 0;
      for (int u = blockIdx.x; u < total; u += gridDim.x) {
        int mt, nt;
        unit_tile(p, u, num_tiles, mt, nt);
        const int g = p.tile_group[mt], row0 = p.tile_row0[mt];
        const bool sh = (g == p.shared_group);
        const CUtensorMap* mb = sh ? &tmBs : &tmB;
        const int wrow = (sh ? 0 : g * p.w_rows) + nt * p.b_row_step;
        bool ok = true;
        for (int kb = 0; kb < p.kb_count; ++kb, ++it) {
          const int s = it % S;
          const uint32_t round = it / S;
          if (p.prefetch > 0 && it + p.prefetch < my_iters) {
            int pkb, pwrow;
            const CUtensorMap* pmb;
            weight_rows(it + p.prefetch, pkb, pwrow, pmb);
            tma_prefetch_l2_2d(pmb, pkb * BK, pwrow, pol_w);
            tma_prefetch_l2_2d(pmb, pkb * BK, pwrow + p.b_row_hi, pol_w);
          }
          if (blockIdx.x == 0 && it == p.stall_iter) {
            ok = false;  // test hook: withhold this stage (no expect_tx, no loads)
            break;
          }
          if (!mbar_wait(&empty[s], (round & 1) ^ 1, abort_flag, p.err, kErrGemmProducerWait, p.wait_limit)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * C::kStageBytes;
          mbar_arrive_expect_tx(&full[s], C::kStageBytes);
#pragma unroll
          for (int pl = 0; pl < PLANES; ++pl)
            tma_load_2d(st + pl * kTileA, &tmA, &full[s], pl * p.plane_stride + kb * BK, row0, pol_a);
          uint8_t* sb = st + PLANES * kTileA;
          tma_load_2d(sb, mb, &full[s], kb * BK, wrow, pol_w);
          tma_load_2d(sb + kTileA, mb, &full[s], kb * BK, wrow + p.b_row_hi, pol_w);
        }
        if (!ok) break;
      }
      // Let every copy this thread issued land before the CTA can exit.
      for (int s = 0; s < S && s < it; ++s) {
        const int last = s + S * ((it - 1 - s) / S);
        mbar_wait_drain(&full[s], (last / S) & 1);
      }
    }
   } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3_f32(BM, BN);
      // Descriptors of every stage's operand tiles, computed once: a K step
      // of 32 bytes inside the 128-byte swizzle row adds 2 (16-byte units) to
      // the start-address field.  Keeps this thread's per-K-block issue short;
      // it shares an SM sub-partition with two epilogue warps.
      uint64_t da[S][PLANES], db[S];
#pragma unroll
      for (int s = 0; s < S; ++s) {
        uint8_t* st = smem + s * C::kStageBytes;
#pragma unroll
        for (int pl = 0; pl < PLANES; ++pl) da[s][pl] = smem_desc_k_sw128(smem_u32(st + pl * kTileA));
        db[s] = smem_desc_k_sw128(smem_u32(st + PLANES * kTileA));
      }
      const uint32_t tmem_d = *reinterpret_cast<volatile const uint32_t*>(tmem_holder);
      int it = 0, acc_it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        for (int kb = 0; kb < p.kb_count; ++kb, ++it, ++acc_it) {
          const int buf = acc_it & 1;
          // The smem stage is normally ready long before the TMEM buffer is
          // released, so its (cheap, satisfied) wait goes first and the
          // buffer wait is the last step before the MMAs.
          const int s = it % S;
          if (!mbar_wait(&full[s], (it / S) & 1, abort_flag, p.err, kErrGemmMmaWait, p.wait_limit)) {
            ok = false;
            break;
          }
          if (!mbar_wait(&pempty[buf], ((acc_it >> 1) & 1) ^ 1, abort_flag, p.err, kErrGemmMmaWait,
                         p.wait_limit)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem_d + buf * BN;
          uint64_t bd = db[0];
          uint64_t ad[PLANES];
#pragma unroll
          for (int ss = 0; ss < S; ++ss)
            if (ss == s) {
              bd = db[ss];
#pragma unroll
              for (int pl = 0; pl < PLANES; ++pl) ad[pl] = da[ss][pl];
            }
#pragma unroll
          for (int pl = 0; pl < PLANES; ++pl) {
#pragma unroll
            for (int ks = 0; ks < BK / UMMA_K; ++ks)
              umma_f8f6f4(d, ad[pl] + 2 * ks, bd + 2 * ks, idesc, (pl | ks) != 0);
          }
          umma_commit(&empty[s]);
          umma_commit(&pfull[buf]);
        }
      }
      // On every exit path, wait (bounded) for this thread's MMAs to finish
      // before the CTA can free TMEM.
      umma_commit(mma_done);
      mbar_wait_drain(mma_done, 0);
    }
   }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(Regs<MODE>::epi));
    // ------------------------------------------------------------ epilogue
    const int ew = warp - kEpiFirstWarp;
    const int q = warp & 3;         // TMEM lane quadrant this warp may access
    const int h = ew >> 2;          // column half
    const int r = q * 32 + lane;    // row within the tile
    const uint32_t lane_base =
        *reinterpret_cast<volatile const uint32_t*>(tmem_holder) + (static_cast<uint32_t>(q * 32) << 16);
    const int wblk = p.w_rows / kBlock;
    int acc_it = 0, unit_i = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total && ok; u += gridDim.x, ++unit_i) {
      int mt, nt;
      unit_tile(p, u, num_tiles, mt, nt);
      const int g = p.tile_group[mt], row0 = p.tile_row0[mt], rows = p.tile_rows[mt];
      const bool valid = r < rows;
      const float* ws = (g == p.shared_group) ? p.sw_scale : p.w_scale + (size_t)g * wblk * p.kb_count;
      // weight-scale rows used by this thread's two column groups
      int blk0, blk1;
      if (MODE == 0) {
        blk0 = nt;                          // gate rows  [nt*128, +128)
        blk1 = p.I / kBlock + nt;           // up rows    [I + nt*128, +128)
      } else {
        blk0 = blk1 = 2 * nt + h;           // output columns [nt*256 + 128h, +128)
      }
      // Scales are prefetched three K blocks ahead (global-load latency is
      // ~1 pipeline iteration under load).  Rows past the tile's valid count
      // read row 0's scale and are never stored.
      const float* a_sc = p.a_scale + row0 + (valid ? r : 0);
      const float* w0p = ws + (size_t)blk0 * p.kb_count;
      const float* w1p = ws + (size_t)blk1 * p.kb_count;
      float acc[128];
#pragma unroll
      for (int i = 0; i < 128; ++i) acc[i] = 0.f;
      const int KB = p.kb_count;
      float as0 = __ldg(a_sc), w00 = __ldg(w0p), w10 = __ldg(w1p);
      float as1 = 0.f, w01 = 0.f, w11 = 0.f, as2 = 0.f, w02 = 0.f, w12 = 0.f;
      if (KB > 1) {
        as1 = __ldg(a_sc + (size_t)p.a_scale_ld);
        w01 = __ldg(w0p + 1);
        w11 = __ldg(w1p + 1);
      }
      if (KB > 2) {
        as2 = __ldg(a_sc + 2 * (size_t)p.a_scale_ld);
        w02 = __ldg(w0p + 2);
        w12 = __ldg(w1p + 2);
      }
      for (int kb = 0; kb < KB; ++kb, ++acc_it) {
        const float f0 = as0 * w00, f1 = as0 * w10;
        as0 = as1; w00 = w01; w10 = w11;
        as1 = as2; w01 = w02; w11 = w12;
        if (kb + 3 < KB) {
          as2 = __ldg(a_sc + (size_t)(kb + 3) * p.a_scale_ld);
          w02 = __ldg(w0p + kb + 3);
          w12 = __ldg(w1p + kb + 3);
        }
        const int buf = acc_it & 1;
        // Every lane waits on the barrier itself and the warp agrees with one
        // vote: no broadcast from a polling lane on this per-K-block path
        // (lane 0 polling, then a shuffle and __syncwarp, made GEMM1 ~5 %
        // slower).  The epilogue waits on the MMA, which waits on the
        // producer, so a lost stage must be reported by the MMA thread and the
        // epilogue must leave through the abort flag (read every 256 polls).
        // The single MMA thread's polls sleep up to the suspend hint each, so
        // its first clock check can come ~256 polls (~0.25 s) into its wait;
        // the 32 lanes here poll far faster.  Their limit is therefore 4x the
        // pipeline limit and never under 2^30 cycles (> 0.5 s).
        const long long epi_limit = p.wait_limit * 4 > (1ll << 30) ? p.wait_limit * 4 : (1ll << 30);
        const int got = __all_sync(0xffffffffu, mbar_wait(&pfull[buf], (acc_it >> 1) & 1, abort_flag, p.err,
                                                          kErrGemmEpilogueWait, epi_limit, 1024u));
        if (!got) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; c += 2) {
          int col0, col1;
          float fa, fb;
          if (MODE == 0) {
            // gate columns (c = 0, 1) then up columns (c = 2, 3)
            col0 = (c < 2) ? (64 * h + 32 * c) : (128 + 64 * h + 32 * (c - 2));
            col1 = col0 + 32;
            fa = fb = (c < 2) ? f0 : f1;
          } else {
            col0 = 128 * h + 32 * c;
            col1 = col0 + 32;
            fa = fb = f0;
          }
          float v0[32], v1[32];
          tmem_ld_32x32b_x32(lane_base + buf * BN + col0, v0);
          tmem_ld_32x32b_x32(lane_base + buf * BN + col1, v1);
          tmem_ld_wait();
          if (c == 2) {
            // The buffer's last columns are in registers: release it to the
            // MMA before these columns' FMAs (shortens the MMA -> promotion ->
            // MMA hand-off by the FMA time).
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&pempty[buf]);
          }
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            ffma2(acc[32 * c + i], acc[32 * c + i + 1], fa, v0[i], v0[i + 1]);
            ffma2(acc[32 * c + 32 + i], acc[32 * c + 33 + i], fb, v1[i], v1[i + 1]);
          }
        }
      }
      if (!ok) break;

      if (MODE == 0) {
        // SwiGLU: C = silu(up) * gate  (flashinfer_baseline.py:157-160)
        float amax = 0.f;
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          const float up = acc[64 + j];
          // silu(up) = up * 1/(1 + e^-up) with the hardware reciprocal (rel.
          // error ~2^-23; C is requantised to e4m3 planes right after, and the
          // IEEE-rounded reciprocal cost ~8k cycles per tile here).  A
          // saturated e^-up gives 1/inf = 0.
          const float cval = up * rcp_approx(1.0f + __expf(-up)) * acc[j];
          acc[j] = cval;
          amax = fmaxf(amax, fabsf(cval));
        }
        float* ax = amax_x + (unit_i & 1) * 256;
        ax[h * 128 + r] = amax;
        named_bar_sync(1, kEpiWarps * 32);
        amax = fmaxf(amax, ax[(1 - h) * 128 + r]);
        const float scale = amax > 0.f ? __fdiv_rn(amax, kFp8Max) : 1.0f;
        const float inv = amax > 0.f ? __fdiv_rn(kFp8Max, amax) : 1.0f;
        if (valid) {
          const size_t row_bytes = (size_t)OUT_PLANES * p.I;
          uint8_t* dst = p.inter + (size_t)(row0 + r) * row_bytes + (size_t)nt * kBlock + 64 * h;
#pragma unroll
          for (int j0 = 0; j0 < 64; j0 += 16) {
            uint32_t w[OUT_PLANES][4];
#pragma unroll
            for (int j = 0; j < 16; j += 2) {
              float x0 = acc[j0 + j] * inv, x1 = acc[j0 + j + 1] * inv;
#pragma unroll
              for (int pl = 0; pl < OUT_PLANES; ++pl) {
                const uint16_t b2 = f2_to_e4m3x2(x0, x1);
                if ((j & 2) == 0)
                  w[pl][j >> 2] = b2;
                else
                  w[pl][j >> 2] |= static_cast<uint32_t>(b2) << 16;
                if (pl + 1 < OUT_PLANES) {
                  const float2 back = e4m3x2_to_f2(b2);
                  x0 -= back.x;
                  x1 -= back.y;
                }
              }
            }
#pragma unroll
            for (int pl = 0; pl < OUT_PLANES; ++pl)
              *reinterpret_cast<uint4*>(dst + (size_t)pl * p.I + j0) = make_uint4(w[pl][0], w[pl][1], w[pl][2], w[pl][3]);
          }
          if (h == 0) p.inter_scale[(size_t)nt * p.inter_scale_ld + row0 + r] = scale;
        }
      } else {
        // Weighted rows are added into their tokens' fp32 output rows.  Lane =
        // row in TMEM, so a direct float4 atomic per lane would touch 32 rows
        // per instruction; instead each 32-row x 16-column chunk goes through
        // shared memory and comes back with 4 lanes per row, so every vector
        // RED covers 64 contiguous bytes of 8 rows.
        float* stage = reinterpret_cast<float*>(smem + C::kRingBytes + 4096) + ew * (32 * 20);
        // With pair_out the row goes to its own grouped row instead (a plain
        // store; the per-token sum happens later in a fixed order).
        const bool slots = p.pair_out != nullptr;
        const int dst_me = valid ? (slots ? row0 + r : p.row_dest[row0 + r]) : -1;
        const float wgt = valid ? p.row_weight[row0 + r] : 0.f;
        int dst_i[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) dst_i[i] = __shfl_sync(0xffffffffu, dst_me, 8 * i + (lane >> 2));
        float* obase = (slots ? p.pair_out : p.out) + (size_t)nt * BN + 128 * h + 4 * (lane & 3);
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
#pragma unroll
          for (int k = 0; k < 4; ++k)
            *reinterpret_cast<float4*>(stage + lane * 20 + 4 * k) =
                make_float4(wgt * acc[16 * ch + 4 * k], wgt * acc[16 * ch + 4 * k + 1], wgt * acc[16 * ch + 4 * k + 2],
                            wgt * acc[16 * ch + 4 * k + 3]);
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int row = 8 * i + (lane >> 2);
            if (dst_i[i] >= 0) {
              const float4 v = *reinterpret_cast<const float4*>(stage + row * 20 + 4 * (lane & 3));
              float4* o = reinterpret_cast<float4*>(obase + (size_t)dst_i[i] * p.H + 16 * ch);
              if (slots)
                *o = v;
              else
                atomicAdd(o, v);
            }
          }
          __syncwarp();
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(*reinterpret_cast<volatile const uint32_t*>(tmem_holder), kTmemCols);
  }
}

// ------------------------------------------------------------------ host
// Test hook state (gemms_test_inject_stall): which GEMM (1 or 2, 0 = none)
// stalls at which K iteration, and the pipeline wait limit in SM cycles.
std::atomic<int> g_stall_gemm{0};
std::atomic<int> g_stall_iter{-1};
std::atomic<long long> g_wait_limit{GEMMS_WAIT_TIMEOUT_CYCLES};

void apply_wait_knobs(GemmParams& p, int gemm) {
  p.wait_limit = g_wait_limit.load(std::memory_order_relaxed);
  p.stall_iter = g_stall_gemm.load(std::memory_order_relaxed) == gemm ? g_stall_iter.load(std::memory_order_relaxed)
                                                                        : -1;
}

// Weight K-blocks a CTA keeps in flight toward L2 beyond its smem ring.  The
// weight stream is DRAM-latency bound (one 32 KB stage per K-block per SM);
// GEMMS_PREFETCH overrides the default for tuning.
// Unit order of the grouped GEMMs: GEMMS_GEMM_UNIT_ORDER=expert puts an
// expert's M tiles side by side (see unit_tile); default: N tiles fastest.
bool expert_unit_order() {
  static const bool v = [] {
    const char* e = std::getenv("GEMMS_GEMM_UNIT_ORDER");
    return e && std::strcmp(e, "expert") == 0;
  }();
  return v;
}

int prefetch_depth() {
  static int depth = -1;
  if (depth < 0) {
    const char* e = getenv("GEMMS_PREFETCH");
    depth = e ? atoi(e) : 0;
    if (depth < 0) depth = 0;
    if (depth > 64) depth = 64;
  }
  return depth;
}

// 2-D uint8 tensor [rows, inner] with a 128x128 box and 128-byte swizzle.
int make_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint64_t row_stride) {
  auto fn = encode_fn();
  if (!fn) return GEMMS_ERR_DRIVER;
  if (!aligned16(base) || (row_stride % 16) || inner % BK) return GEMMS_ERR_ALIGN;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_stride};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), static_cast<cuuint32_t>(BM)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? GEMMS_OK : GEMMS_ERR_DRIVER;
}

template <int MODE, int PLANES, int OUT_PLANES>
int launch_kernel(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& bs, const GemmParams& p,
                  int max_units, cudaStream_t s) {
  auto kern = grouped_gemm_kernel<MODE, PLANES, OUT_PLANES>;
  constexpr int smem = Cfg<PLANES>::kSmemBytes;
  // The shared-memory opt-in is per device: one bit per device (per template
  // instance) that has been given it.
  static std::atomic<unsigned long long> attr_set{0};
  int dev = 0;
  GEMMS_CUDA_TRY(cudaGetDevice(&dev));
  const unsigned long long bit = dev < 64 ? (1ull << dev) : 0ull;
  if (!bit || !(attr_set.load(std::memory_order_relaxed) & bit)) {
    GEMMS_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr_set.fetch_or(bit, std::memory_order_relaxed);
  }
  const int grid = std::max(1, std::min(gemm_ctas(), max_units));
  kern<<<grid, kThreads, smem, s>>>(a, b, bs, p);
  GEMMS_CUDA_TRY(cudaGetLastError());
  return GEMMS_OK;
}

}  // namespace

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

int launch_gemm1(const Gemm1Args& a, cudaStream_t s) {
  if (a.H % BK || a.I % BK) return GEMMS_ERR_SHAPE;
  if (a.planes < 2 || a.planes > 3) return GEMMS_ERR_SHAPE;
  CUtensorMap ma, mb, mbs;
  int rc;
  if ((rc = make_map(&ma, a.a, a.H, a.a_rows, a.H))) return rc;
  if ((rc = make_map(&mb, a.w13, a.H, (uint64_t)a.E_local * 2 * a.I, a.H))) return rc;
  if (a.sw13) {
    if ((rc = make_map(&mbs, a.sw13, a.H, 2ull * a.I, a.H))) return rc;
  } else {
    mbs = mb;
  }
  GemmParams p{};
  p.tile_group = a.g.tile_group;
  p.tile_row0 = a.g.tile_row0;
  p.tile_rows = a.g.tile_rows;
  p.num_tiles = a.g.num_tiles;
  p.max_tiles = a.g.max_tiles;
  p.shared_group = a.sw13 ? a.g.shared_group : -1;
  p.n_tiles = a.I / kBlock;
  p.kb_count = a.H / BK;
  p.plane_stride = 0;
  p.w_rows = 2 * a.I;
  p.b_row_step = kBlock;
  p.b_row_hi = a.I;
  p.prefetch = prefetch_depth();
  p.group_tile0 = expert_unit_order() ? a.g.group_tile0 : nullptr;
  p.a_scale = a.a_scale;
  p.a_scale_ld = a.a_scale_ld;
  p.w_scale = a.w13_scale;
  p.sw_scale = a.sw13_scale;
  p.inter = a.inter;
  p.inter_scale = a.inter_scale;
  p.inter_scale_ld = a.inter_scale_ld;
  p.I = a.I;
  p.H = a.H;
  p.err = a.err;
  apply_wait_knobs(p, 1);
  const int max_units = a.g.max_tiles * p.n_tiles;
  if (a.planes == 2) return launch_kernel<0, 1, 2>(ma, mb, mbs, p, max_units, s);
  return launch_kernel<0, 1, 3>(ma, mb, mbs, p, max_units, s);
}

int launch_gemm2(const Gemm2Args& a, cudaStream_t s) {
  if (a.H % BN || a.I % BK) return GEMMS_ERR_SHAPE;
  if (a.planes < 2 || a.planes > 3) return GEMMS_ERR_SHAPE;
  CUtensorMap ma, mb, mbs;
  int rc;
  if ((rc = make_map(&ma, a.inter, (uint64_t)a.planes * a.I, a.a_rows, (uint64_t)a.planes * a.I))) return rc;
  if ((rc = make_map(&mb, a.w2, a.I, (uint64_t)a.E_local * a.H, a.I))) return rc;
  if (a.sw2) {
    if ((rc = make_map(&mbs, a.sw2, a.I, (uint64_t)a.H, a.I))) return rc;
  } else {
    mbs = mb;
  }
  GemmParams p{};
  p.tile_group = a.g.tile_group;
  p.tile_row0 = a.g.tile_row0;
  p.tile_rows = a.g.tile_rows;
  p.num_tiles = a.g.num_tiles;
  p.max_tiles = a.g.max_tiles;
  p.shared_group = a.sw2 ? a.g.shared_group : -1;
  p.n_tiles = a.H / BN;
  p.kb_count = a.I / BK;
  p.plane_stride = a.I;
  p.w_rows = a.H;
  p.b_row_step = BN;
  p.b_row_hi = kBlock;
  p.prefetch = prefetch_depth();
  p.group_tile0 = expert_unit_order() ? a.g.group_tile0 : nullptr;
  p.a_scale = a.inter_scale;
  p.a_scale_ld = a.inter_scale_ld;
  p.w_scale = a.w2_scale;
  p.sw_scale = a.sw2_scale;
  p.row_dest = a.row_dest;
  p.row_weight = a.row_weight;
  p.out = a.out;
  p.pair_out = a.pair_out;
  p.H = a.H;
  p.I = a.I;
  p.err = a.err;
  apply_wait_knobs(p, 2);
  const int max_units = a.g.max_tiles * p.n_tiles;
  if (a.planes == 2) return launch_kernel<1, 2, 1>(ma, mb, mbs, p, max_units, s);
  return launch_kernel<1, 3, 1>(ma, mb, mbs, p, max_units, s);
}

// Upper bound on the persistent GEMM grid (0 = one CTA per SM).  The grouped
// GEMMs hold every SM they get for their whole run, so a collective kernel
// launched on another stream only progresses on SMs left free; the
// expert-parallel path lowers the bound while a GEMM overlaps an all-to-all.
std::atomic<int> g_gemm_cta_limit{0};

int gemm_ctas() {
  const int lim = g_gemm_cta_limit.load(std::memory_order_relaxed);
  return lim > 0 ? std::min(lim, num_sms()) : num_sms();
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    n = v;
  }
  return n;
}

}  // namespace gemms

extern "C" int gemms_test_inject_stall(int32_t gemm, int32_t k_iteration, int64_t wait_limit_cycles) {
  if (gemm < 0 || gemm > 2 || wait_limit_cycles < 0) return GEMMS_ERR_ARG;
  if (gemm == 0) {
    gemms::g_stall_gemm.store(0);
    gemms::g_stall_iter.store(-1);
    gemms::g_wait_limit.store(GEMMS_WAIT_TIMEOUT_CYCLES);
    return GEMMS_OK;
  }
  if (k_iteration < 0) return GEMMS_ERR_ARG;
  gemms::g_wait_limit.store(wait_limit_cycles > 0 ? wait_limit_cycles : GEMMS_WAIT_TIMEOUT_CYCLES);
  gemms::g_stall_iter.store(k_iteration);
  gemms::g_stall_gemm.store(gemm);
  return GEMMS_OK;
}

extern "C" int gemms_set_gemm_ctas(int32_t max_ctas) {
  if (max_ctas < 0) return GEMMS_ERR_ARG;
  return gemms::g_gemm_cta_limit.exchange(max_ctas);
}
