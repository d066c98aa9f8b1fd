/*
 * gemms_moe.h -- C ABI of the B200-native DeepSeek-V3 FP8 MoE layer.
 *
 * Plain pointers and sizes only; the caller owns every buffer.  All entry
 * points are stream-ordered (nothing synchronises the host unless the name
 * says so) and return 0 on success or a negative GEMMS_ERR_* code.  No entry
 * point calls exit().
 *
 * Reference interfaces replaced (plops655/GEMMS):
 *   gemms_moe_fwd        <- launch_persistent_moe_v2(...)      persistent_kernel2.cu:896-910
 *                           and the operator run(...)           flashinfer_baseline.py:5-16
 *   gemms_route          <- routing_topk_kernel                 persistent_kernel2.cu:153-299
 *   gemms_expert_ffn     <- persistent_gemm_kernel phases 1+2   persistent_kernel2.cu:388-890
 *   gemms_moe_workspace_size <- ScratchOffsets2 / compute_scratch_offsets2
 *                                                               persistent_kernel2.cu:32-67
 *   gemms_strerror       <- CUDA_CHECK's message+exit           common.h:8-15
 */
#ifndef GEMMS_MOE_H_
#define GEMMS_MOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cudaStream_t without pulling in the CUDA headers. */
typedef struct CUstream_st* gemms_stream_t;

enum {
  GEMMS_OK = 0,
  GEMMS_ERR_SHAPE = -1,      /* unsupported or inconsistent geometry            */
  GEMMS_ERR_ALIGN = -2,      /* a pointer is not 16-byte aligned                */
  GEMMS_ERR_WORKSPACE = -3,  /* workspace missing or smaller than required      */
  GEMMS_ERR_CUDA = -4,       /* a CUDA runtime call failed                      */
  GEMMS_ERR_TIMEOUT = -5,    /* a device-side wait gave up (error word set)     */
  GEMMS_ERR_DRIVER = -6,     /* cuTensorMapEncodeTiled unavailable or failed    */
  GEMMS_ERR_DEVICE = -7,     /* current device is not sm_100                    */
  GEMMS_ERR_ARG = -8,        /* a required pointer is NULL                      */
  GEMMS_ERR_CAPACITY = -9    /* a size exceeds a fixed capacity of this entry   */
};

/* Bits of the device error word (gemms_moe_check, gemms_moe_check_noalloc). */
enum {
  GEMMS_FLAG_PRODUCER_WAIT = 1 << 0,  /* GEMM TMA producer gave up on a free stage */
  GEMMS_FLAG_MMA_WAIT = 1 << 1,       /* GEMM MMA thread gave up on data / TMEM    */
  GEMMS_FLAG_EPILOGUE_WAIT = 1 << 2,  /* GEMM epilogue gave up on a partial        */
  GEMMS_FLAG_BAD_EXPERT = 1 << 3,     /* a received row named a non-local expert   */
  GEMMS_FLAG_ROW_OVERFLOW = 1 << 4    /* more M tiles than the workspace holds     */
};

/* Activation input formats. */
enum {
  GEMMS_INPUT_BF16 = 0,      /* x bf16 [T,H]; quantised per 1x128 inside        */
  GEMMS_INPUT_FP8 = 1        /* e4m3 [T,H] + fp32 scale [H/128, T] (run())      */
};

typedef struct {
  int32_t T;                    /* tokens                                          */
  int32_t H;                    /* hidden size, multiple of 128                    */
  int32_t I;                    /* expert intermediate size, multiple of 128       */
  int32_t E;                    /* routed experts (width of the logits)            */
  int32_t E_local;              /* experts whose weights are passed                */
  int32_t local_expert_offset;  /* global id of local expert 0                     */
  int32_t n_group;              /* routing groups; E/n_group in {2,4,8,16,32}      */
  int32_t topk_group;           /* groups kept per token                           */
  int32_t top_k;                /* experts per token, <= 16                        */
  int32_t has_shared;           /* 1: a shared expert (weight 1.0) is applied      */
  int32_t input_mode;           /* GEMMS_INPUT_*                                   */
  int32_t bias_bf16;            /* 1: routing_bias is bf16, 0: fp32                */
  int32_t inter_planes;         /* e4m3 planes of the SwiGLU intermediate: 2 or 3  */
  float routed_scaling_factor;
  int32_t deterministic;        /* 1: bit-reproducible combine -- each (token,     */
                                /* expert) result row is stored, then summed per   */
                                /* token in slot order (k routed, then shared);    */
                                /* 0: fp32 vector atomics (faster, order-dependent */
                                /* in the last bits); 1 adds R*H*4 workspace bytes */
} GemmsMoeShape;

typedef struct {
  GemmsMoeShape shape;
  const float* routing_logits;      /* fp32 [T, E]; NULL: computed from router_w   */
  const void* routing_bias;         /* fp32 or bf16 [E]                            */
  const void* hidden_bf16;          /* bf16 [T, H]       (GEMMS_INPUT_BF16)        */
  const void* hidden_fp8;           /* e4m3 [T, H]       (GEMMS_INPUT_FP8)         */
  const float* hidden_scale;        /* fp32 [H/128, T]   (GEMMS_INPUT_FP8)         */
  const void* w13;                  /* e4m3 [E_local, 2I, H]                       */
  const float* w13_scale;           /* fp32 [E_local, 2I/128, H/128]               */
  const void* w2;                   /* e4m3 [E_local, H, I]                        */
  const float* w2_scale;            /* fp32 [E_local, H/128, I/128]                */
  const void* shared_w13;           /* e4m3 [2I, H]          (has_shared)          */
  const float* shared_w13_scale;    /* fp32 [2I/128, H/128]  (has_shared)          */
  const void* shared_w2;            /* e4m3 [H, I]           (has_shared)          */
  const float* shared_w2_scale;     /* fp32 [H/128, I/128]   (has_shared)          */
  void* out;                        /* bf16 [T, H], written (not accumulated)      */
  int32_t* topk_idx_out;            /* optional int32 [T, top_k] (NULL: skip)      */
  float* topk_w_out;                /* optional fp32 [T, top_k]                    */
  int32_t* expert_counts_out;       /* optional int32 [E_local]                    */
  void* const* profile_events;      /* optional: 3 cudaEvent_t recorded on the     */
                                    /* stream before GEMM1, between GEMM1 and      */
                                    /* GEMM2, and after GEMM2 (kernel timing)      */
  const float* router_w;            /* fp32 [E, H]: with routing_logits NULL and   */
                                    /* GEMMS_INPUT_BF16, logits = x . router_w^T   */
                                    /* on the tensor cores (bf16 hi/lo split)      */
  float* logits_out;                /* optional fp32 [T, E]: the logits used       */
  const void* residual;             /* optional bf16 [T, H]: out = bf16(residual + */
                                    /* layer), one rounding (the decoder's         */
                                    /* residual add after the MoE block)           */
} GemmsMoeArgs;

/* Bytes of device workspace gemms_moe_fwd needs for this shape. */
size_t gemms_moe_workspace_size(const GemmsMoeShape* shape);

/* Batches of at most max_t tokens (<= 2) run the two expert GEMMs on the CUDA
 * cores as weight streams (with so few rows per expert the tensor-core GEMMs
 * are bound by their per-K-block chain, not by HBM); 0 keeps every batch on
 * the tensor cores.  Default 1 (faster than the tensor cores at T=1, slower at
 * T=4, measured on one box), or GEMMS_DECODE_MAX_T at library load.  The
 * workspace size depends on it: query gemms_moe_workspace_size after setting
 * it.  Returns the previous value, or GEMMS_ERR_ARG if negative.  No
 * counterpart in the reference. */
int gemms_set_decode_max_t(int32_t max_t);

/* Full layer forward: route -> permute(+quant) -> GEMM1+SwiGLU -> GEMM2 ->
 * weighted combine (+ shared expert) -> bf16.  Workspace must be 256-byte
 * aligned and at least gemms_moe_workspace_size() bytes; the contents need no
 * initialisation.  Concurrent calls need distinct workspaces. */
int gemms_moe_fwd(const GemmsMoeArgs* args, void* workspace, size_t ws_bytes, gemms_stream_t stream);

/* gemms_moe_fwd without a caller workspace, for callers that cannot allocate
 * device memory where they run the layer (plugin hosts that provide a stream
 * but no allocator, runtimes that forbid allocations once serving starts).
 * No counterpart in the reference.  Scratch is a fixed 16 MiB device array
 * inside this library, held by every GPU that loads it until process exit;
 * shapes whose gemms_moe_workspace_size() exceeds 16 MiB are rejected with
 * GEMMS_ERR_CAPACITY (DeepSeek-V3 shapes with a shared expert: up to 119
 * tokens when the layer computes the router logits from bf16 activations,
 * 126 with given logits and FP8 activations).  The first call on a device looks up the array's device address
 * (make it before any stream capture).  All calls share the array: calls that
 * overlap on the GPU (other streams, other host threads) race.  Allocates
 * nothing. */
int gemms_moe_fwd_noalloc(const GemmsMoeArgs* args, gemms_stream_t stream);

/* Router GEMM alone: logits fp32 [T, E] = x bf16 [T, H] . router_w fp32
 * [E, H]^T (H a multiple of 64, E <= 256).  T > 128: x . hi^T + x . lo^T
 * with router_w = hi + lo + r split into two bf16 planes (|r| <= 2^-16 |w|)
 * and fp32 accumulation on the tensor cores; T <= 128 (decode): fp32 FMAs on
 * the CUDA cores over router_w as given.  Deterministic (split-K partials are
 * summed in a fixed order).  Workspace: gemms_router_workspace_size().
 * No counterpart in the reference, which takes logits as input
 * (flashinfer_baseline.py:6). */
size_t gemms_router_workspace_size(int32_t T, int32_t H, int32_t E);
int gemms_router_logits(const void* x_bf16, const float* router_w, int32_t T, int32_t H, int32_t E, float* logits,
                        void* workspace, size_t ws_bytes, gemms_stream_t stream);

/* Per-1x128 activation quantisation: x bf16 [T, H] -> xq e4m3 [T, H] and
 * xq_scale fp32 [H/128, T] (the transposed layout of the reference's
 * hidden_states_scale, flashinfer_baseline.py:59,72), scale = amax/448 (1.0
 * for an all-zero block), xq = e4m3(x / scale) rounded to nearest even with
 * IEEE division.  No counterpart in the reference (its run() takes quantised
 * activations). */
int gemms_quantize_1x128(const void* x_bf16, int32_t T, int32_t H, void* xq, float* xq_scale,
                         gemms_stream_t stream);

/* The step before the layer: RMSNorm fused with the per-1x128 quantisation.
 * h bf16 [T, H] (H a multiple of 128), weight bf16 (weight_bf16 = 1) or fp32
 * [H] ->  y = weight * bf16(h * rsqrt(mean(h^2) + eps)) rounded to bf16 (the
 * DeepSeek-V3 RMSNorm) into y_bf16 [T, H] (optional: the router GEMM's
 * input), and its 1x128 e4m3 quantisation into xq [T, H] + xq_scale
 * [H/128, T] (optional, as gemms_quantize_1x128: the experts' input with
 * GEMMS_INPUT_FP8).  No counterpart in the reference (its operator starts
 * from quantised activations, flashinfer_baseline.py:5-16). */
int gemms_rmsnorm_quant(const void* h_bf16, const void* weight, int32_t weight_bf16, float eps, int32_t T,
                        int32_t H, void* y_bf16, void* xq, float* xq_scale, gemms_stream_t stream);

/* Router only (for tests and expert-parallel dispatch): fp32 logits [T,E] +
 * bias -> topk_idx int32 [T,top_k] (descending biased score), topk_w fp32
 * [T,top_k] (normalised, times the scaling factor), and counts int32 [E]
 * (histogram over all E experts; must be zeroed by the caller). */
int gemms_route(const float* logits, const void* bias, int32_t bias_bf16, int32_t T, int32_t E,
                int32_t n_group, int32_t topk_group, int32_t top_k, float routed_scaling_factor,
                int32_t* topk_idx, float* topk_w, int32_t* counts, gemms_stream_t stream);

/* Expert FFN over rows that are already grouped by expert (expert-parallel
 * receive side): rows [0, R) hold e4m3 activations [R, H] with scales
 * [H/128, R] (row-major per 128-column block, leading dimension R);
 * expert_counts[E_local] (device) gives how many consecutive rows belong to
 * each local expert, in order.  Row r's result times row_weight[r] is added
 * into out_f32[row_dest[r], :] (fp32 [n_dest, H], accumulated, not zeroed).
 * Workspace: gemms_expert_ffn_workspace_size(). */
size_t gemms_expert_ffn_workspace_size(int32_t R_max, int32_t H, int32_t I, int32_t E_local,
                                       int32_t inter_planes);
int gemms_expert_ffn(const void* rows_fp8, const float* rows_scale, int32_t R_max,
                     const int32_t* expert_counts, const int32_t* row_dest, const float* row_weight,
                     int32_t H, int32_t I, int32_t E_local, int32_t inter_planes,
                     const void* w13, const float* w13_scale, const void* w2, const float* w2_scale,
                     float* out_f32, void* workspace, size_t ws_bytes, gemms_stream_t stream);

/* ---- expert parallel (rank r owns experts [r*E_local, (r+1)*E_local)) ----
 * No counterpart in the reference, which has only the local_expert_offset
 * slicing hook (flashinfer_baseline.py:132-138); the all-to-alls are NCCL
 * calls made by the host (gemms_b200/ep.py).
 *
 * Packed dispatch row: e4m3 [H] | fp32 scales [H/128] | int32 expert ids
 * [top_k] (-1 = not on the destination) | fp32 weights [top_k], padded to 16 B. */
size_t gemms_ep_row_bytes(int32_t H, int32_t top_k);

/* topk_idx/topk_w [T, top_k] (global ids) + x bf16 [T, H] ->
 * send_counts int32 [2, world] (zeroed here): [0][d] rows sent to rank d and
 * [1][d] routed (token, expert) pairs they carry for d's experts (the sizes
 * of d's grouped rows), send_row_of [T, world] (-1 = not sent),
 * send_buf [<= T*min(world,top_k), row_bytes] grouped by destination in token
 * order, and the token-major quantised rows xq [T, H] + xq_scale [H/128, T]. */
int gemms_ep_dispatch(const int32_t* topk_idx, const float* topk_w, const void* x_bf16, int32_t T, int32_t H,
                      int32_t top_k, int32_t world, int32_t E_local, int32_t* send_counts, int32_t* send_row_of,
                      void* send_buf, void* xq, float* xq_scale, gemms_stream_t stream);

/* Received packed rows [R, row_bytes] -> out_rows fp32 [R, H] (overwritten):
 * each row's results summed over its experts on this rank, times weights.
 * P_max bounds the (row, local expert) pairs the rows name (the sum over
 * sources of their send_counts[1][this rank]); the workspace holds that many
 * grouped rows.  Rows beyond it are not computed and set GEMMS_FLAG_ROW_OVERFLOW
 * in the workspace's error word (gemms_moe_check). */
size_t gemms_ep_ffn_workspace_size(int32_t R_max, int32_t P_max, int32_t H, int32_t I, int32_t E_local,
                                   int32_t top_k, int32_t inter_planes);
int gemms_ep_expert_ffn(const void* recv_buf, int32_t R, int32_t P_max, int32_t H, int32_t I, int32_t top_k,
                        int32_t E_local, int32_t local_expert_offset, int32_t inter_planes, const void* w13,
                        const float* w13_scale, const void* w2, const float* w2_scale, float* out_rows,
                        void* workspace, size_t ws_bytes, gemms_stream_t stream);

/* Packed combine row: fp16 [H] holding value / 2^e | fp32 2^e | pad to 16 B,
 * with 2^e the power of two that puts max|row| / 2^e in [2^14, 2^15) (e = 0
 * for zero or non-finite rows): the scaling is exact, only fp16 rounding is
 * added.  Halves the bytes of the combine all-to-all against fp32 rows. */
size_t gemms_ep_back_row_bytes(int32_t H);

/* out_rows fp32 [R, H] (gemms_ep_expert_ffn) -> packed [R, back_row_bytes]. */
int gemms_ep_pack_back(const float* rows, int32_t R, int32_t H, void* packed, gemms_stream_t stream);

/* out bf16 [T, H] = acc fp32 [T, H] + sum over d of the packed row
 * back_packed[send_row_of[t, d]] (fp16 x 2^e), gathered in rank order. */
int gemms_ep_combine(const float* acc, const void* back_packed, const int32_t* send_row_of, int32_t T, int32_t H,
                     int32_t world, void* out_bf16, gemms_stream_t stream);

/* As gemms_ep_combine, but destination d's packed rows are read in place: the
 * row for (t, d) is row send_row_of[t, d] + row_add[d] of the buffer at
 * row_base[d] (host arrays of `world` entries; 16-byte aligned device
 * addresses, which may be other GPUs' memory mapped into this process, e.g.
 * the peer pointers of a symmetric allocation, read over NVLink).  The caller
 * guarantees that every row read lies inside its buffer, that its writers
 * have finished before this call's kernel starts, and that they do not write
 * it again until the kernel has completed.  No counterpart in the reference. */
int gemms_ep_combine_rows(const float* acc, const void* const* row_base, const int32_t* row_add,
                          const int32_t* send_row_of, int32_t T, int32_t H, int32_t world, void* out_bf16,
                          gemms_stream_t stream);

/* ---- device-driven exchange (no host read of counts) ----
 * Replaces the count exchange and the dispatch all-to-all: every rank owns an
 * exchange region in memory that all ranks can address (a symmetric
 * allocation; its peer pointers are read over NVLink):
 *   [0, 256)    int32 counts [2][world], written by gemms_ep_dispatch as its
 *               send_counts
 *   [256, ...)  send rows [send_cap, row_bytes], gemms_ep_dispatch's send_buf
 * gemms_ep_region_bytes gives the size.  After a barrier that orders every
 * rank's dispatch before this call, gemms_ep_pull reads all ranks' counts and
 * copies the rows sent to `rank` from their regions into recv_buf
 * [recv_cap, row_bytes] (received rows ordered by source rank, then by the
 * source's token order), and writes the plan to info (int32 [128], device):
 *   info[0]       R, rows received (0 when a flag is set)
 *   info[1]       P, routed (row, local expert) pairs they carry
 *   info[2]       flags: 1 = more than recv_cap rows were sent to this rank,
 *                 2 = a region's counts exceed send_cap or are negative;
 *                 nothing is copied when set
 *   info[8 + s]   first received row from rank s (s = 0..world)
 *   info[48 + s]  where this rank's rows start among rank s's send rows
 *   info[88 + d]  offset for gemms_ep_combine_peer: this rank's combine row
 *                 for (t, d) is row send_row_of[t, d] + info[88 + d] of d's
 *                 packed combine rows
 * region[s] are the `world` region addresses (host array).  The caller keeps
 * every region unwritten until all ranks' pulls of this call have completed.
 * No counterpart in the reference (its only distributed hook is
 * local_expert_offset, flashinfer_baseline.py:132-138). */
size_t gemms_ep_region_bytes(int32_t send_cap, int32_t H, int32_t top_k);
int gemms_ep_pull(const void* const* region, int32_t rank, int32_t world, int32_t H, int32_t top_k,
                  int32_t send_cap, int32_t recv_cap, void* recv_buf, int32_t* info, gemms_stream_t stream);

/* gemms_ep_expert_ffn over the first info[0] of R_cap received rows (the row
 * count is read on the device; launches are sized for R_cap). */
int gemms_ep_expert_ffn_dev(const void* recv_buf, int32_t R_cap, const int32_t* info, int32_t P_max, int32_t H,
                            int32_t I, int32_t top_k, int32_t E_local, int32_t local_expert_offset,
                            int32_t inter_planes, const void* w13, const float* w13_scale, const void* w2,
                            const float* w2_scale, float* out_rows, void* workspace, size_t ws_bytes,
                            gemms_stream_t stream);

/* gemms_ep_pack_back over the first info[0] of R_cap rows. */
int gemms_ep_pack_back_dev(const float* rows, int32_t R_cap, const int32_t* info, int32_t H, void* packed,
                           gemms_stream_t stream);

/* gemms_ep_combine_rows with the row offsets taken from gemms_ep_pull's info
 * (info[88 + d]) on the device; every rank's packed combine rows hold
 * recv_cap rows, and a row index outside [0, recv_cap) (only after a pull
 * that raised a flag) is skipped, not read. */
int gemms_ep_combine_peer(const float* acc, const void* const* row_base, const int32_t* info,
                          const int32_t* send_row_of, int32_t T, int32_t H, int32_t world, int32_t recv_cap,
                          void* out_bf16, gemms_stream_t stream);

/* acc fp32 [T, H] += this rank's combine rows read in place from every
 * destination's region (the same rows and offsets as gemms_ep_combine_peer),
 * with fp32 vector atomics, so that other kernels (the shared expert's GEMMs)
 * may add into acc at the same time; then gemms_f32_to_bf16 casts the sum. */
int gemms_ep_gather_add_peer(float* acc, const void* const* row_base, const int32_t* info,
                             const int32_t* send_row_of, int32_t T, int32_t H, int32_t world, int32_t recv_cap,
                             gemms_stream_t stream);

/* out bf16 [n] = in fp32 [n] rounded to nearest even; n a multiple of 4. */
int gemms_f32_to_bf16(const float* in, void* out_bf16, size_t n, gemms_stream_t stream);

/* CTAs of gemms_ep_pull's row copy for later calls (0 = two per SM, the
 * default); returns the previous value, or GEMMS_ERR_ARG if negative. */
int gemms_ep_set_pull_ctas(int32_t ctas);

/* Bounds the grid of the persistent grouped-GEMM kernels to max_ctas CTAs
 * (0 = one per SM, the default) for launches made after the call, from any
 * thread.  Returns the previous bound, or GEMMS_ERR_ARG for a negative value.
 * The GEMMs keep every SM they are given for their whole run, so a collective
 * on another stream (the expert-parallel all-to-alls) only progresses on SMs
 * left free.  No counterpart in the reference. */
int gemms_set_gemm_ctas(int32_t max_ctas);

/* Reads and clears the device error word kept in a gemms_moe_fwd workspace.
 * Synchronises the stream.  *flags receives the raw bit set (0 = clean). */
int gemms_moe_check(void* workspace, gemms_stream_t stream, int32_t* flags);

/* gemms_moe_check for the fixed scratch array of gemms_moe_fwd_noalloc on the
 * current device: reads and clears its device error word (synchronises the
 * stream).  A device-side wait that gave up inside a no-alloc call is only
 * visible here; the next no-alloc call clears the word.  No counterpart in the
 * reference. */
int gemms_moe_check_noalloc(gemms_stream_t stream, int32_t* flags);

/* Test hook (not for production use): from the next launch on, the producer
 * of CTA 0 of grouped GEMM `gemm` (1 or 2) stops issuing at K iteration
 * `k_iteration`, leaving no copy in flight, and every pipeline wait of that
 * GEMM gives up after `wait_limit_cycles` SM cycles (0: the default ~4 s).
 * The MMA thread's wait for the missing stage then runs out: the kernel sets
 * bit 1 (MMA wait) of the device error word, lets its issued work drain,
 * frees its tensor memory and returns, so the context stays usable and
 * gemms_moe_check reports GEMMS_ERR_TIMEOUT.  gemm = 0 restores the default
 * (no stall, default limit).  Replaces, for testing, the unbounded spins of
 * persistent_kernel2.cu:747-757 (no counterpart). */
int gemms_test_inject_stall(int32_t gemm, int32_t k_iteration, int64_t wait_limit_cycles);

/* Test hook (not for production use): where a gemms_moe_fwd workspace of
 * this shape keeps, after a call, the layer's expert-grouped activation rows
 * (e4m3 [R, H], R = T*top_k, + T rows of the shared expert), their fp32
 * 1x128 scales ([H/128][scale_ld], grouped row fastest), the (token, slot) ->
 * grouped row map (int32 [T, top_k], -1 for an expert outside the local
 * range) and the per-group first rows (int32 [E_local + 1 (+1)], the shared
 * expert's group last), as byte offsets from the workspace base.  Lets a test
 * compare the rows the permute step wrote with a CPU quantisation.  The
 * decode path (T at most gemms_set_decode_max_t's limit) writes no grouped
 * rows.  No counterpart in the reference. */
int gemms_test_workspace_regions(const GemmsMoeShape* shape, size_t* rows_off, size_t* scale_off,
                                 int32_t* scale_ld, size_t* pair_row_off, size_t* offsets_off);

/* Static description of an error code. */
const char* gemms_strerror(int code);

/* Library version string. */
const char* gemms_version(void);

#ifdef __cplusplus
}
#endif

#endif /* GEMMS_MOE_H_ */
