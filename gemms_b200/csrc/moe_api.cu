// moe_api.cu -- the extern "C" boundary (include/gemms_moe.h).
//
// Replaces launch_persistent_moe_v2 (persistent_kernel2.cu:896-1010), which
// cudaMallocAsync's and frees its scratch on every call and exits the process
// on any CUDA error (common.h:8-15).  Here the caller passes a workspace once
// sized by gemms_moe_workspace_size(); every step is stream-ordered and errors
// come back as GEMMS_ERR_* codes.
#include "common.cuh"

#include <atomic>
#include <cstdlib>

#include <algorithm>

namespace gemms {
namespace {

struct FwdLayout {
  int T, K, H, I, E_loc, shared, planes;
  int R_max, groups, max_tiles, scale_ld;
  size_t err, counts, topk_idx, topk_w, pair_row, offsets, tile_group, tile_row0, tile_rows, num_tiles;
  size_t row_token, row_weight, a_rows, a_scale, inter, inter_scale, out_acc, pair_out, total;
  int det;  // deterministic combine: per-row results in pair_out, summed per token in slot order
  int decode_rows;  // > 0: expert GEMMs on the CUDA cores (decode.cu) for tiles of <= decode_rows rows
  size_t dec_inter;  // fp32 SwiGLU output [R_max, I] of the decode path
  RouterPlan router;
  size_t router_planes, router_partials;  // router GEMM scratch (GEMMS_INPUT_BF16 only)
  size_t head_bytes;  // [0, head_bytes) is zeroed each call (error word + counts)
};

// Largest batch that takes the CUDA-core expert GEMMs: GEMMS_DECODE_MAX_T at
// load time (default 1: measured faster than the tensor cores at T=1 and
// slower at T=4 on the same box; 0 keeps every batch on the tensor cores),
// changed by gemms_set_decode_max_t (at most kDecodeMaxRows).
std::atomic<int> g_decode_t_limit{[] {
  const char* e = std::getenv("GEMMS_DECODE_MAX_T");
  const int x = e ? std::atoi(e) : 1;
  return std::max(0, std::min(x, kDecodeMaxRows));
}()};
int decode_t_limit() { return g_decode_t_limit.load(std::memory_order_relaxed); }

FwdLayout fwd_layout(const GemmsMoeShape& s) {
  FwdLayout L{};
  L.T = s.T;
  L.K = s.top_k;
  L.H = s.H;
  L.I = s.I;
  L.E_loc = s.E_local;
  L.shared = s.has_shared ? 1 : 0;
  L.planes = s.inter_planes == 0 ? 2 : s.inter_planes;
  L.R_max = s.T * s.top_k + (L.shared ? s.T : 0);
  L.groups = s.E_local + L.shared;
  L.max_tiles = cdiv(L.R_max, kBlock) + L.groups;
  L.scale_ld = static_cast<int>(align_up(std::max(L.R_max, 1), 32));
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align_up(o + bytes, 256);
    return at;
  };
  L.err = take(64);
  L.counts = take(sizeof(int32_t) * std::max(L.E_loc, 1));
  L.head_bytes = o;
  L.topk_idx = take(sizeof(int32_t) * (size_t)L.T * L.K);
  L.topk_w = take(sizeof(float) * (size_t)L.T * L.K);
  L.pair_row = take(sizeof(int32_t) * (size_t)L.T * L.K);
  L.offsets = take(sizeof(int32_t) * 2 * (L.groups + 1));  // offsets, then first tile per group
  L.tile_group = take(sizeof(int32_t) * L.max_tiles);
  L.tile_row0 = take(sizeof(int32_t) * L.max_tiles);
  L.tile_rows = take(sizeof(int32_t) * L.max_tiles);
  L.num_tiles = take(sizeof(int32_t));
  L.row_token = take(sizeof(int32_t) * (size_t)std::max(L.R_max, 1));
  L.row_weight = take(sizeof(float) * (size_t)std::max(L.R_max, 1));
  L.a_rows = take((size_t)std::max(L.R_max, 1) * L.H);
  L.a_scale = take(sizeof(float) * (size_t)(L.H / kBlock) * L.scale_ld);
  L.inter = take((size_t)std::max(L.R_max, 1) * L.planes * L.I);
  L.inter_scale = take(sizeof(float) * (size_t)(L.I / kBlock) * L.scale_ld);
  L.decode_rows = 0;
  if (s.T >= 1 && s.T <= decode_t_limit() && decode_shape_ok(s.H, s.I))
    L.decode_rows = s.T <= 1 ? 1 : 2;  // tiles hold <= T rows (routed and shared)
  if (L.decode_rows) L.dec_inter = take(sizeof(float) * (size_t)std::max(L.R_max, 1) * L.I);
  L.det = s.deterministic ? 1 : 0;
  if (L.det)
    L.pair_out = take(sizeof(float) * (size_t)std::max(L.R_max, 1) * L.H);
  else
    L.out_acc = take(sizeof(float) * (size_t)L.T * L.H);
  if (s.input_mode == GEMMS_INPUT_BF16) {
    L.router = router_plan(s.T, s.H, s.E);
    L.router_planes = L.router.split_bytes ? take(L.router.split_bytes) : 0;
    L.router_partials = take(L.router.partial_bytes);
  }
  L.total = o;
  return L;
}

int check_shape(const GemmsMoeShape& s) {
  if (s.T < 0 || s.H <= 0 || s.I <= 0 || s.E <= 0 || s.E_local < 0) return GEMMS_ERR_SHAPE;
  if (s.H % 256 || s.I % kBlock) return GEMMS_ERR_SHAPE;
  if (s.E > 256 || (s.E > 32 && s.E % 32)) return GEMMS_ERR_SHAPE;
  if (s.n_group <= 0 || s.E % s.n_group) return GEMMS_ERR_SHAPE;
  const int gs = s.E / s.n_group;
  if (gs < 2 || gs > 32 || (gs & (gs - 1))) return GEMMS_ERR_SHAPE;
  if (s.topk_group < 1 || s.topk_group > s.n_group) return GEMMS_ERR_SHAPE;
  if (s.top_k < 1 || s.top_k > 16 || s.top_k > s.topk_group * gs) return GEMMS_ERR_SHAPE;
  if (s.input_mode != GEMMS_INPUT_BF16 && s.input_mode != GEMMS_INPUT_FP8) return GEMMS_ERR_SHAPE;
  const int planes = s.inter_planes == 0 ? 2 : s.inter_planes;
  if (planes < 2 || planes > 3) return GEMMS_ERR_SHAPE;
  if ((long long)s.T * s.top_k + s.T > (1ll << 30)) return GEMMS_ERR_SHAPE;
  return GEMMS_OK;
}

int check_device() {
  static int ok = -1;
  if (ok < 0) {
    int dev = 0, major = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return GEMMS_ERR_CUDA;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return GEMMS_ERR_CUDA;
    ok = (major == 10) ? 1 : 0;
  }
  return ok ? GEMMS_OK : GEMMS_ERR_DEVICE;
}

template <class T>
T* at(void* ws, size_t off) {
  return reinterpret_cast<T*>(static_cast<char*>(ws) + off);
}

}  // namespace
}  // namespace gemms

using namespace gemms;

extern "C" {

const char* gemms_version(void) { return "gemms_b200 0.1 (sm_100a)"; }

const char* gemms_strerror(int code) {
  switch (code) {
    case GEMMS_OK: return "ok";
    case GEMMS_ERR_SHAPE: return "unsupported or inconsistent shape";
    case GEMMS_ERR_ALIGN: return "pointer or stride not 16-byte aligned";
    case GEMMS_ERR_WORKSPACE: return "workspace missing or too small";
    case GEMMS_ERR_CUDA: return "CUDA runtime error";
    case GEMMS_ERR_TIMEOUT: return "a device-side wait timed out";
    case GEMMS_ERR_DRIVER: return "cuTensorMapEncodeTiled unavailable or failed";
    case GEMMS_ERR_DEVICE: return "current device is not an sm_100 (B200) GPU";
    case GEMMS_ERR_ARG: return "a required pointer is NULL";
    case GEMMS_ERR_CAPACITY: return "size exceeds a fixed capacity of this entry point";
    default: return "unknown error";
  }
}

int gemms_set_decode_max_t(int32_t max_t) {
  if (max_t < 0) return GEMMS_ERR_ARG;
  return gemms::g_decode_t_limit.exchange(std::min<int>(max_t, gemms::kDecodeMaxRows));
}

size_t gemms_moe_workspace_size(const GemmsMoeShape* shape) {
  if (!shape || check_shape(*shape) != GEMMS_OK) return 0;
  return fwd_layout(*shape).total;
}

int gemms_moe_fwd(const GemmsMoeArgs* args, void* workspace, size_t ws_bytes, gemms_stream_t stream_) {
  if (!args) return GEMMS_ERR_ARG;
  const GemmsMoeShape& s = args->shape;
  int rc = check_shape(s);
  if (rc) return rc;
  if ((rc = check_device())) return rc;
  const FwdLayout L = fwd_layout(s);
  if (!workspace || ws_bytes < L.total) return GEMMS_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 255u) return GEMMS_ERR_ALIGN;
  const bool gemm_router = args->routing_logits == nullptr;
  if (!args->routing_bias || !args->out) return GEMMS_ERR_ARG;
  if (gemm_router && (s.input_mode != GEMMS_INPUT_BF16 || !args->router_w || !args->hidden_bf16))
    return GEMMS_ERR_ARG;
  if (gemm_router && !aligned16(args->router_w)) return GEMMS_ERR_ALIGN;
  if (s.E_local > 0 && (!args->w13 || !args->w13_scale || !args->w2 || !args->w2_scale)) return GEMMS_ERR_ARG;
  if (s.input_mode == GEMMS_INPUT_BF16 && !args->hidden_bf16) return GEMMS_ERR_ARG;
  if (s.input_mode == GEMMS_INPUT_FP8 && (!args->hidden_fp8 || !args->hidden_scale)) return GEMMS_ERR_ARG;
  if (s.has_shared && (!args->shared_w13 || !args->shared_w13_scale || !args->shared_w2 || !args->shared_w2_scale))
    return GEMMS_ERR_ARG;
  for (const void* p : {args->hidden_bf16, args->hidden_fp8, args->w13, args->w2, args->shared_w13, args->shared_w2,
                        static_cast<const void*>(args->out)})
    if (p && !aligned16(p)) return GEMMS_ERR_ALIGN;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
  if (s.T == 0) return GEMMS_OK;

  void* ws = workspace;
  int* err = at<int>(ws, L.err);
  GEMMS_CUDA_TRY(cudaMemsetAsync(ws, 0, L.head_bytes, st));
  // (the decode front kernel zeroes the accumulator itself)
  const bool fused_front = L.decode_rows > 0;
  if (!L.det && !fused_front)
    GEMMS_CUDA_TRY(cudaMemsetAsync(at<char>(ws, L.out_acc), 0, sizeof(float) * (size_t)L.T * L.H, st));

  RouteArgs ra{};
  if (gemm_router) {
    RouterGemmArgs rg{};
    rg.plan = L.router;
    rg.x = static_cast<const __nv_bfloat16*>(args->hidden_bf16);
    rg.router_w = args->router_w;
    rg.T = s.T;
    rg.H = s.H;
    rg.E = s.E;
    rg.planes = L.router.split_bytes ? at<__nv_bfloat16>(ws, L.router_planes) : nullptr;
    rg.partials = at<float>(ws, L.router_partials);
    rg.err = err;
    if ((rc = launch_router_gemm(rg, st))) return rc;
    ra.partials = rg.partials;
    ra.n_partials = L.router.splits;
    ra.logits_out = args->logits_out;
  } else {
    ra.logits = args->routing_logits;
    if (args->logits_out)
      GEMMS_CUDA_TRY(cudaMemcpyAsync(args->logits_out, args->routing_logits, sizeof(float) * (size_t)s.T * s.E,
                                     cudaMemcpyDeviceToDevice, st));
  }
  ra.bias = args->routing_bias;
  ra.bias_bf16 = s.bias_bf16;
  ra.T = s.T;
  ra.E = s.E;
  ra.n_group = s.n_group;
  ra.topk_group = s.topk_group;
  ra.top_k = s.top_k;
  ra.rsf = s.routed_scaling_factor;
  ra.local_offset = s.local_expert_offset;
  ra.E_local = s.E_local;
  ra.topk_idx = at<int32_t>(ws, L.topk_idx);
  ra.topk_w = at<float>(ws, L.topk_w);
  ra.counts = at<int32_t>(ws, L.counts);
  ra.pair_row = at<int32_t>(ws, L.pair_row);

  PlanArgs pa{};
  pa.counts = at<int32_t>(ws, L.counts);
  pa.E_local = s.E_local;
  pa.shared_rows = L.shared ? s.T : 0;
  pa.offsets = at<int32_t>(ws, L.offsets);
  pa.tile_group = at<int32_t>(ws, L.tile_group);
  pa.tile_row0 = at<int32_t>(ws, L.tile_row0);
  pa.tile_rows = at<int32_t>(ws, L.tile_rows);
  pa.num_tiles = at<int32_t>(ws, L.num_tiles);
  pa.group_tile0 = pa.offsets + (L.groups + 1);
  pa.max_tiles = L.max_tiles;
  pa.row_capacity = L.R_max;
  pa.err = err;

  AssignArgs sa{};
  sa.topk_idx = ra.topk_idx;
  sa.topk_w = ra.topk_w;
  sa.T = s.T;
  sa.top_k = s.top_k;
  sa.local_offset = s.local_expert_offset;
  sa.E_local = s.E_local;
  sa.offsets = pa.offsets;
  sa.row_token = at<int32_t>(ws, L.row_token);
  sa.row_weight = at<float>(ws, L.row_weight);
  sa.pair_row = ra.pair_row;
  sa.shared_rows = pa.shared_rows;
  sa.row_capacity = L.R_max;
  if (fused_front && decode_front_ok(ra, pa)) {
    if ((rc = launch_decode_front(ra, pa, sa, L.det ? nullptr : at<float>(ws, L.out_acc), (size_t)L.T * L.H, st)))
      return rc;
  } else {
    if (fused_front && !L.det)
      GEMMS_CUDA_TRY(cudaMemsetAsync(at<char>(ws, L.out_acc), 0, sizeof(float) * (size_t)L.T * L.H, st));
    if ((rc = launch_route(ra, st))) return rc;
    if ((rc = launch_plan(pa, st))) return rc;
    if ((rc = launch_assign(sa, st))) return rc;
  }

  PermuteArgs qa{};
  qa.mode = s.input_mode;
  qa.x_bf16 = static_cast<const __nv_bfloat16*>(args->hidden_bf16);
  qa.x_fp8 = static_cast<const uint8_t*>(args->hidden_fp8);
  qa.x_scale = args->hidden_scale;
  qa.T = s.T;
  qa.H = s.H;
  qa.top_k = s.top_k;
  qa.pair_row = ra.pair_row;
  qa.shared_row0 = L.shared ? pa.offsets + s.E_local : nullptr;
  qa.rows_fp8 = at<uint8_t>(ws, L.a_rows);
  qa.rows_scale = at<float>(ws, L.a_scale);
  qa.scale_ld = L.scale_ld;
  // the CUDA-core decode GEMM1 reads the input rows itself (no permuted copy)
  DecodeSrc dsrc{};
  if (L.decode_rows) {
    dsrc.row_token = sa.row_token;
    dsrc.x_bf16 = s.input_mode == GEMMS_INPUT_BF16 ? qa.x_bf16 : nullptr;
    dsrc.x_fp8 = qa.x_fp8;
    dsrc.x_scale = qa.x_scale;
    dsrc.T = s.T;
  } else if ((rc = launch_permute(qa, st))) {
    return rc;
  }

  GemmGroupsArgs gg{};
  gg.tile_group = pa.tile_group;
  gg.tile_row0 = pa.tile_row0;
  gg.tile_rows = pa.tile_rows;
  gg.num_tiles = pa.num_tiles;
  gg.group_tile0 = pa.group_tile0;
  gg.max_tiles = L.max_tiles;
  gg.shared_group = L.shared ? s.E_local : -1;

  Gemm1Args g1{};
  g1.g = gg;
  g1.a = qa.rows_fp8;
  g1.a_rows = L.R_max;
  g1.a_scale = qa.rows_scale;
  g1.a_scale_ld = L.scale_ld;
  g1.w13 = static_cast<const uint8_t*>(args->w13);
  g1.w13_scale = args->w13_scale;
  g1.E_local = std::max(s.E_local, 1);
  g1.sw13 = L.shared ? static_cast<const uint8_t*>(args->shared_w13) : nullptr;
  g1.sw13_scale = args->shared_w13_scale;
  g1.H = s.H;
  g1.I = s.I;
  g1.planes = L.planes;
  g1.inter = at<uint8_t>(ws, L.inter);
  g1.inter_scale = at<float>(ws, L.inter_scale);
  g1.inter_scale_ld = L.scale_ld;
  g1.err = err;
  if (!g1.w13) g1.w13 = g1.sw13;
  cudaEvent_t const* evs = reinterpret_cast<cudaEvent_t const*>(args->profile_events);
  float* dec_inter = L.decode_rows ? at<float>(ws, L.dec_inter) : nullptr;
  if (evs) GEMMS_CUDA_TRY(cudaEventRecord(evs[0], st));
  if ((rc = L.decode_rows ? launch_decode_gemm1(g1, dec_inter, L.decode_rows, &dsrc, st) : launch_gemm1(g1, st))) return rc;
  if (evs) GEMMS_CUDA_TRY(cudaEventRecord(evs[1], st));

  Gemm2Args g2{};
  g2.g = gg;
  g2.inter = g1.inter;
  g2.a_rows = L.R_max;
  g2.inter_scale = g1.inter_scale;
  g2.inter_scale_ld = L.scale_ld;
  g2.w2 = static_cast<const uint8_t*>(args->w2);
  g2.w2_scale = args->w2_scale;
  g2.E_local = std::max(s.E_local, 1);
  g2.sw2 = L.shared ? static_cast<const uint8_t*>(args->shared_w2) : nullptr;
  g2.sw2_scale = args->shared_w2_scale;
  g2.H = s.H;
  g2.I = s.I;
  g2.planes = L.planes;
  g2.row_dest = sa.row_token;
  g2.row_weight = sa.row_weight;
  g2.out = L.det ? nullptr : at<float>(ws, L.out_acc);
  g2.pair_out = L.det ? at<float>(ws, L.pair_out) : nullptr;
  g2.err = err;
  if (!g2.w2) g2.w2 = g2.sw2;
  if ((rc = L.decode_rows ? launch_decode_gemm2(g2, dec_inter, L.decode_rows, st) : launch_gemm2(g2, st))) return rc;
  if (evs) GEMMS_CUDA_TRY(cudaEventRecord(evs[2], st));

  if (L.det) {
    if ((rc = launch_combine_slots(g2.pair_out, ra.pair_row, s.T, s.top_k, s.H, qa.shared_row0,
                                   static_cast<const __nv_bfloat16*>(args->residual),
                                   static_cast<__nv_bfloat16*>(args->out), nullptr, nullptr, st)))
      return rc;
  } else if ((rc = launch_to_bf16(g2.out, static_cast<__nv_bfloat16*>(args->out), (size_t)s.T * s.H,
                                  static_cast<const __nv_bfloat16*>(args->residual), st))) {
    return rc;
  }

  if (args->topk_idx_out)
    GEMMS_CUDA_TRY(cudaMemcpyAsync(args->topk_idx_out, ra.topk_idx, sizeof(int32_t) * (size_t)s.T * s.top_k,
                                   cudaMemcpyDeviceToDevice, st));
  if (args->topk_w_out)
    GEMMS_CUDA_TRY(cudaMemcpyAsync(args->topk_w_out, ra.topk_w, sizeof(float) * (size_t)s.T * s.top_k,
                                   cudaMemcpyDeviceToDevice, st));
  if (args->expert_counts_out && s.E_local > 0)
    GEMMS_CUDA_TRY(cudaMemcpyAsync(args->expert_counts_out, ra.counts, sizeof(int32_t) * s.E_local,
                                   cudaMemcpyDeviceToDevice, st));
  return GEMMS_OK;
}

int gemms_test_workspace_regions(const GemmsMoeShape* shape, size_t* rows_off, size_t* scale_off,
                                  int32_t* scale_ld, size_t* pair_row_off, size_t* offsets_off) {
  if (!shape || !rows_off || !scale_off || !scale_ld || !pair_row_off || !offsets_off) return GEMMS_ERR_ARG;
  int rc = check_shape(*shape);
  if (rc) return rc;
  const FwdLayout L = fwd_layout(*shape);
  *rows_off = L.a_rows;
  *scale_off = L.a_scale;
  *scale_ld = L.scale_ld;
  *pair_row_off = L.pair_row;
  *offsets_off = L.offsets;
  return GEMMS_OK;
}

int gemms_moe_check(void* workspace, gemms_stream_t stream_, int32_t* flags) {
  if (!workspace || !flags) return GEMMS_ERR_ARG;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
  int32_t v = 0;
  GEMMS_CUDA_TRY(cudaMemcpyAsync(&v, workspace, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
  GEMMS_CUDA_TRY(cudaStreamSynchronize(st));
  *flags = v;
  if (v) {
    GEMMS_CUDA_TRY(cudaMemsetAsync(workspace, 0, sizeof(int32_t), st));
    return GEMMS_ERR_TIMEOUT;
  }
  return GEMMS_OK;
}

int gemms_route(const float* logits, const void* bias, int32_t bias_bf16, int32_t T, int32_t E, int32_t n_group,
                int32_t topk_group, int32_t top_k, float routed_scaling_factor, int32_t* topk_idx, float* topk_w,
                int32_t* counts, gemms_stream_t stream_) {
  GemmsMoeShape s{};
  s.T = T;
  s.H = 256;
  s.I = 128;
  s.E = E;
  s.E_local = E;
  s.n_group = n_group;
  s.topk_group = topk_group;
  s.top_k = top_k;
  s.inter_planes = 2;
  int rc = check_shape(s);
  if (rc) return rc;
  if ((rc = check_device())) return rc;
  if (!logits || !bias || !topk_idx || !topk_w) return GEMMS_ERR_ARG;
  RouteArgs ra{};
  ra.logits = logits;
  ra.bias = bias;
  ra.bias_bf16 = bias_bf16;
  ra.T = T;
  ra.E = E;
  ra.n_group = n_group;
  ra.topk_group = topk_group;
  ra.top_k = top_k;
  ra.rsf = routed_scaling_factor;
  ra.local_offset = 0;
  ra.E_local = counts ? E : 0;
  ra.topk_idx = topk_idx;
  ra.topk_w = topk_w;
  ra.counts = counts;
  ra.pair_row = nullptr;
  return launch_route(ra, reinterpret_cast<cudaStream_t>(stream_));
}

}  // extern "C"

namespace gemms {
namespace {
struct FfnLayout {
  int groups, max_tiles, scale_ld;
  size_t err, offsets, tile_group, tile_row0, tile_rows, num_tiles, inter, inter_scale, total;
};
FfnLayout ffn_layout(int R_max, int H, int I, int E_local, int planes) {
  (void)H;
  FfnLayout L{};
  L.groups = E_local;
  L.max_tiles = cdiv(std::max(R_max, 1), kBlock) + E_local;
  L.scale_ld = static_cast<int>(align_up(std::max(R_max, 1), 32));
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align_up(o + bytes, 256);
    return at;
  };
  L.err = take(64);
  L.offsets = take(sizeof(int32_t) * 2 * (L.groups + 1));  // offsets, then first tile per group
  L.tile_group = take(sizeof(int32_t) * L.max_tiles);
  L.tile_row0 = take(sizeof(int32_t) * L.max_tiles);
  L.tile_rows = take(sizeof(int32_t) * L.max_tiles);
  L.num_tiles = take(sizeof(int32_t));
  L.inter = take((size_t)std::max(R_max, 1) * planes * I);
  L.inter_scale = take(sizeof(float) * (size_t)(I / kBlock) * L.scale_ld);
  L.total = o;
  return L;
}
}  // namespace
}  // namespace gemms

extern "C" {

size_t gemms_expert_ffn_workspace_size(int32_t R_max, int32_t H, int32_t I, int32_t E_local, int32_t inter_planes) {
  if (R_max < 0 || H <= 0 || I <= 0 || E_local <= 0 || H % 256 || I % kBlock) return 0;
  const int planes = inter_planes == 0 ? 2 : inter_planes;
  if (planes < 2 || planes > 3) return 0;
  return ffn_layout(R_max, H, I, E_local, planes).total;
}

int gemms_expert_ffn(const void* rows_fp8, const float* rows_scale, int32_t R_max, const int32_t* expert_counts,
                     const int32_t* row_dest, const float* row_weight, int32_t H, int32_t I, int32_t E_local,
                     int32_t inter_planes, const void* w13, const float* w13_scale, const void* w2,
                     const float* w2_scale, float* out_f32, void* workspace, size_t ws_bytes,
                     gemms_stream_t stream_) {
  if (R_max < 0 || H <= 0 || I <= 0 || E_local <= 0 || H % 256 || I % kBlock) return GEMMS_ERR_SHAPE;
  const int planes = inter_planes == 0 ? 2 : inter_planes;
  if (planes < 2 || planes > 3) return GEMMS_ERR_SHAPE;
  int rc;
  if ((rc = check_device())) return rc;
  if (!rows_fp8 || !rows_scale || !expert_counts || !row_dest || !row_weight || !w13 || !w13_scale || !w2 ||
      !w2_scale || !out_f32)
    return GEMMS_ERR_ARG;
  const FfnLayout L = ffn_layout(R_max, H, I, E_local, planes);
  if (!workspace || ws_bytes < L.total) return GEMMS_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 255u) return GEMMS_ERR_ALIGN;
  if (R_max == 0) return GEMMS_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
  void* ws = workspace;
  int* err = at<int>(ws, L.err);
  GEMMS_CUDA_TRY(cudaMemsetAsync(ws, 0, 64, st));

  PlanArgs pa{};
  pa.counts = expert_counts;
  pa.E_local = E_local;
  pa.shared_rows = 0;
  pa.offsets = at<int32_t>(ws, L.offsets);
  pa.tile_group = at<int32_t>(ws, L.tile_group);
  pa.tile_row0 = at<int32_t>(ws, L.tile_row0);
  pa.tile_rows = at<int32_t>(ws, L.tile_rows);
  pa.num_tiles = at<int32_t>(ws, L.num_tiles);
  pa.group_tile0 = pa.offsets + (L.groups + 1);
  pa.max_tiles = L.max_tiles;
  pa.row_capacity = std::max(R_max, 1);
  pa.err = err;
  if ((rc = launch_plan(pa, st))) return rc;

  GemmGroupsArgs gg{};
  gg.tile_group = pa.tile_group;
  gg.tile_row0 = pa.tile_row0;
  gg.tile_rows = pa.tile_rows;
  gg.num_tiles = pa.num_tiles;
  gg.group_tile0 = pa.group_tile0;
  gg.max_tiles = L.max_tiles;
  gg.shared_group = -1;

  Gemm1Args g1{};
  g1.g = gg;
  g1.a = static_cast<const uint8_t*>(rows_fp8);
  g1.a_rows = R_max;
  g1.a_scale = rows_scale;
  g1.a_scale_ld = R_max;
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
  g2.a_rows = R_max;
  g2.inter_scale = g1.inter_scale;
  g2.inter_scale_ld = L.scale_ld;
  g2.w2 = static_cast<const uint8_t*>(w2);
  g2.w2_scale = w2_scale;
  g2.E_local = E_local;
  g2.H = H;
  g2.I = I;
  g2.planes = planes;
  g2.row_dest = row_dest;
  g2.row_weight = row_weight;
  g2.out = out_f32;
  g2.err = err;
  return launch_gemm2(g2, st);
}

}  // extern "C"
