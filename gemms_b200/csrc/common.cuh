// common.cuh -- shared definitions of the MoE kernels and their host launchers.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cstdint>
#include <cstddef>

#include <cudaTypedefs.h>

#include "gemms_moe.h"

namespace gemms {

constexpr int kBlock = 128;          // quantisation block (1x128 activations, 128x128 weights)
constexpr float kFp8Max = 448.0f;    // largest finite e4m3 magnitude

// Device error word bits (OR-ed by kernels, read by gemms_moe_check).
enum : int {
  kErrGemmProducerWait = GEMMS_FLAG_PRODUCER_WAIT,
  kErrGemmMmaWait = GEMMS_FLAG_MMA_WAIT,
  kErrGemmEpilogueWait = GEMMS_FLAG_EPILOGUE_WAIT,
  kErrBadExpertIndex = GEMMS_FLAG_BAD_EXPERT,
  kErrRowOverflow = GEMMS_FLAG_ROW_OVERFLOW,
};

#define GEMMS_CUDA_TRY(expr)                         \
  do {                                               \
    cudaError_t _e = (expr);                         \
    if (_e != cudaSuccess) return GEMMS_ERR_CUDA;    \
  } while (0)

__host__ __device__ inline int cdiv(int a, int b) { return (a + b - 1) / b; }
__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---- internal launchers (stream-ordered, return GEMMS_* codes) ----------
struct RouteArgs {
  const float* logits;        // fp32 [T, E], or nullptr when `partials` is given
  const float* partials;      // fp32 [n_partials][T][E] router-GEMM split-K partials, summed in order
  int n_partials;
  float* logits_out;          // optional fp32 [T, E]: the summed logits (partials path only)
  const void* bias;
  int bias_bf16;
  int T, E, n_group, topk_group, top_k;
  float rsf;
  int local_offset, E_local;  // histogram only counts experts in [local_offset, local_offset+E_local)
  int32_t* topk_idx;          // [T, top_k]
  float* topk_w;              // [T, top_k]
  int32_t* counts;            // [E_local]
  int32_t* pair_row;          // optional [T, top_k], set to -1 (filled later by assign)
};
int launch_route(const RouteArgs& a, cudaStream_t s);

// Builds per-group row offsets and the 128-row M-tile list.
// groups = E_local (+1 if a shared expert is appended with `shared_rows` rows).
struct PlanArgs {
  const int32_t* counts;  // [E_local]
  int E_local;
  int shared_rows;        // 0: no shared group
  int32_t* offsets;       // [groups + 1]
  int32_t* tile_group;    // [max_tiles]
  int32_t* tile_row0;
  int32_t* tile_rows;
  int32_t* num_tiles;     // [1]
  int32_t* group_tile0;   // [groups + 1] first M tile of each group (+ total), optional
  int max_tiles;
  int row_capacity;       // grouped rows the buffers hold: more rows -> error word, no tiles
  int* err;
};
int launch_plan(const PlanArgs& a, cudaStream_t s);

// Deterministic (token-ordered) row assignment within each local expert.
struct AssignArgs {
  const int32_t* topk_idx;
  const float* topk_w;
  int T, top_k, local_offset, E_local;
  int idx_stride;          // elements between consecutive tokens' ids / weights (0: top_k)
  const int32_t* offsets;
  int32_t* row_token;     // [rows]
  float* row_weight;      // [rows]
  int32_t* pair_row;      // [T, top_k]
  int shared_rows;         // >0: rows offsets[E_local] + t get token t, weight 1
  int row_capacity;       // rows at or past it are not written (plan_kernel reports the overflow)
  const int32_t* T_dev;   // when set, only tokens t < min(T, *T_dev) (a count made on the device)
};
int launch_assign(const AssignArgs& a, cudaStream_t s);

// Decode-sized batches (T <= 4): route + plan + assign in one launch, same
// results as launch_route, launch_plan and launch_assign in sequence.
bool decode_front_ok(const RouteArgs& ra, const PlanArgs& pa);
// zero_buf (optional, zero_n floats) is cleared by the same kernel.
int launch_decode_front(const RouteArgs& ra, const PlanArgs& pa, const AssignArgs& sa, float* zero_buf,
                        size_t zero_n, cudaStream_t s);

// Gather (and for bf16 input, quantise per 1x128) activation rows into the
// expert-grouped operand: rows_fp8 [R, H], rows_scale [H/128, ld].
struct PermuteArgs {
  int mode;                        // GEMMS_INPUT_BF16 / GEMMS_INPUT_FP8
  const __nv_bfloat16* x_bf16;     // [T, H]
  const uint8_t* x_fp8;            // [T, H]
  const float* x_scale;            // [H/128, T] (or strided, see below)
  int T, H, top_k;
  long long x_row_stride;          // bytes between fp8 input rows (0: H)
  long long scale_kb_stride;       // floats between 128-column blocks of x_scale (0: T)
  long long scale_t_stride;        // floats between tokens of x_scale (0: 1)
  const int32_t* pair_row;         // [T, top_k] (-1 = not local)
  const int32_t* shared_row0;      // device int (nullptr: none); token t also goes to row *shared_row0 + t
  uint8_t* rows_fp8;
  float* rows_scale;
  int scale_ld;
  const int32_t* T_dev;            // when set, only tokens t < *T_dev (a count made on the device)
};
int launch_permute(const PermuteArgs& a, cudaStream_t s);

// Token-major per-1x128 quantisation: bf16 [T, H] -> e4m3 [T, H] + fp32 scale [H/128, T].
int launch_quantize(const __nv_bfloat16* x, int T, int H, uint8_t* xq, float* xq_scale, cudaStream_t s);

// fp32 [n] (+ optional bf16 residual [n]) -> bf16 [n], one rounding
int launch_to_bf16(const float* in, __nv_bfloat16* out, size_t n, const __nv_bfloat16* residual, cudaStream_t s);

// Grouped block-scaled FP8 GEMMs.
struct GemmGroupsArgs {
  const int32_t* tile_group;
  const int32_t* tile_row0;
  const int32_t* tile_rows;
  const int32_t* num_tiles;
  const int32_t* group_tile0;  // [groups + 1] (plan_kernel): lets the GEMMs order units expert by expert
  int max_tiles;
  int shared_group;  // group index that uses the shared expert's weights (-1: none)
};

struct Gemm1Args {
  GemmGroupsArgs g;
  const uint8_t* a;  int a_rows;  const float* a_scale; int a_scale_ld;    // [R, H], [H/128, ld]
  const uint8_t* w13; const float* w13_scale; int E_local;                 // [E_local, 2I, H]
  const uint8_t* sw13; const float* sw13_scale;                            // shared [2I, H]
  int H, I;
  int planes;                                                               // 2 or 3
  uint8_t* inter; float* inter_scale; int inter_scale_ld;                   // [R, planes*I], [I/128, ld]
  int* err;
};
int launch_gemm1(const Gemm1Args& a, cudaStream_t s);

struct Gemm2Args {
  GemmGroupsArgs g;
  const uint8_t* inter; int a_rows; const float* inter_scale; int inter_scale_ld;
  const uint8_t* w2; const float* w2_scale; int E_local;                   // [E_local, H, I]
  const uint8_t* sw2; const float* sw2_scale;                              // shared [H, I]
  int H, I, planes;
  const int32_t* row_dest; const float* row_weight;                        // [R]
  float* out;                                                               // [n_dest, H] fp32 (+=)
  float* pair_out;  // when set: weighted row r stored to pair_out[r] ([R, H] fp32), out unused
  int* err;
};
int launch_gemm2(const Gemm2Args& a, cudaStream_t s);

// Decode-sized batches (decode.cu): the two expert GEMMs on the CUDA cores for
// tiles of at most max_rows (<= kDecodeMaxRows) rows (with more rows per
// expert the FMA work per weight byte makes the tensor cores faster); GEMM1 writes the SwiGLU
// output in fp32 to inter [R, I], GEMM2 reads it (same Gemm*Args as the
// tensor-core path; the planes / inter / inter_scale fields are unused).
constexpr int kDecodeMaxRows = 2;
bool decode_shape_ok(int H, int I);
// With row_token set, GEMM1 reads its activation rows straight from the
// layer's input (token row_token[grouped row]; bf16 quantised per 1x128 as
// permute_kernel does, or e4m3 + [H/128, T] scales) instead of g1.a / a_scale.
struct DecodeSrc {
  const int32_t* row_token;
  const __nv_bfloat16* x_bf16;
  const uint8_t* x_fp8;
  const float* x_scale;
  int T;
};
int launch_decode_gemm1(const Gemm1Args& g1, float* inter, int max_rows, const DecodeSrc* src, cudaStream_t s);
int launch_decode_gemm2(const Gemm2Args& g2, const float* inter, int max_rows, cudaStream_t s);

// Deterministic combine: out[t] = round(residual[t] + sum over j < K of
// pair_out[pair_row[t, j]] (rows < 0 skipped) + pair_out[*shared_row0 + t]),
// added in that order in fp32; bf16 out (residual optional) or fp32 out.
int launch_combine_slots(const float* pair_out, const int32_t* pair_row, int T, int K, int H,
                         const int32_t* shared_row0, const __nv_bfloat16* residual, __nv_bfloat16* out_bf16,
                         float* out_f32, const int32_t* T_dev, cudaStream_t s);

// Router GEMM (router_gemm.cu): logits = x . router_w^T via a bf16 hi/lo split.
struct RouterPlan {
  int simt;          // 1: CUDA-core fp32 path (decode-sized T), no weight planes
  int Np;            // E rounded up to 16 (MMA N)
  int KB;            // 64-element K blocks
  int kb_per_split;
  int splits;        // split-K factor (partials summed by route_kernel / launch_sum_partials)
  size_t split_bytes;    // bf16 planes [2][Np][H]
  size_t partial_bytes;  // fp32 [splits][T][E]
};
RouterPlan router_plan(int T, int H, int E);
struct RouterGemmArgs {
  RouterPlan plan;
  const __nv_bfloat16* x;  // [T, H]
  const float* router_w;   // [E, H]
  int T, H, E;
  __nv_bfloat16* planes;   // workspace, plan.split_bytes
  float* partials;         // workspace, plan.partial_bytes
  int* err;
};
int launch_router_gemm(const RouterGemmArgs& a, cudaStream_t s);
int launch_sum_partials(const float* partials, int splits, int T, int E, float* logits, cudaStream_t s);

// cuTensorMapEncodeTiled through the runtime's driver entry point (nullptr if unavailable).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn();

int num_sms();
int gemm_ctas();  // persistent GEMM grid bound (gemms_set_gemm_ctas)

}  // namespace gemms
