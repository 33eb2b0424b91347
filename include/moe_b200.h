/*
 * moe_b200.h -- C ABI of the B200 (sm_100a) MoE / QMoE hot path.
 *
 * The library libmoe_b200.so implements the com.microsoft MoE and QMoE contrib
 * operators (opset 1) as hand-written CUDA for sm_100a.  Every entry point takes
 * plain pointers and sizes, returns a status code and never throws; the message of
 * the last failure on the calling thread is available from moe_b200_last_error().
 *
 * Mapping to the reference plugin (MooreThreads/onnxruntime-musa, paths relative to
 * its root):
 *   - the per-op kernel object (create / compute / release) replaces what
 *     ONNX_OPERATOR_VERSIONED_KERNEL_EX registers and OpKernelBase<Derived> runs
 *     (musa/ep/src/kernels/utils.h:144-223, kernels/shared_inc/kernel_base.h:33-97);
 *   - the runtime block replaces the MUSA runtime calls behind device discovery,
 *     the allocator, the sync stream and data transfer
 *     (musa/ep/src/ep_factory.cc:389-455, ep_allocator.h:86-278,
 *      ep_stream.cc:30-185, ep_data_transfer.cc:108-227).
 * Status codes are the numeric values of OrtErrorCode so a plugin can pass them to
 * OrtApi::CreateStatus unchanged; element types are ONNX TensorProto codes.
 */
#ifndef MOE_B200_H_
#define MOE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MOE_B200_ABI_VERSION 1

/* Status codes (values of OrtErrorCode). */
enum {
  MOE_B200_OK = 0,
  MOE_B200_FAIL = 1,
  MOE_B200_INVALID_ARGUMENT = 2,
  MOE_B200_NOT_IMPLEMENTED = 9,
  MOE_B200_EP_FAIL = 11
};

/* Element types (ONNX TensorProto.DataType). */
enum {
  MOE_B200_FLOAT = 1,
  MOE_B200_UINT8 = 2,
  MOE_B200_INT32 = 6,
  MOE_B200_FLOAT16 = 10,
  MOE_B200_BFLOAT16 = 16
};

/* activation_type attribute values. */
enum {
  MOE_B200_ACT_RELU = 0,
  MOE_B200_ACT_GELU = 1,
  MOE_B200_ACT_SILU = 2,
  MOE_B200_ACT_IDENTITY = 3,
  MOE_B200_ACT_SWIGLU = 4
};

/* Attributes of one MoE / QMoE node (the com.microsoft schema's attribute set). */
typedef struct moe_b200_attrs {
  int32_t activation_type;          /* MOE_B200_ACT_* */
  int32_t k;                        /* experts per token */
  int32_t normalize_routing_weights;
  int32_t use_sparse_mixer;         /* 1: sparse-mixer top-2 routing (k must be 2;
                                       normalize_routing_weights is then ignored) */
  int32_t swiglu_fusion;            /* 0: fc3 is the linear half; 1 interleaved; 2 halves */
  float swiglu_limit;               /* +inf disables clamping */
  float activation_alpha;
  float activation_beta;
  int32_t expert_weight_bits;       /* 0 for MoE; 4 or 8 for QMoE */
  int32_t block_size;               /* QMoE: 0 = one scale per output row */
} moe_b200_attrs;

/* Shapes of one call.  Weights are [num_experts, N, K], K contiguous. */
typedef struct moe_b200_problem {
  int64_t num_rows;        /* T: tokens (rows of input) */
  int64_t hidden_size;     /* H */
  int64_t inter_size;      /* I: width of the activation fed to fc2 */
  int64_t num_experts;     /* E */
  int32_t dtype;           /* element type of input/router/output (and MoE weights) */
  int32_t has_fc3;
  moe_b200_attrs attrs;
} moe_b200_problem;

/* Device pointers of one call; unused optional inputs are NULL. */
typedef struct moe_b200_tensors {
  const void* input;         /* [T, H] */
  const void* router_probs;  /* [T, E] router logits */
  const void* fc1_weights;   /* MoE: [E, I or 2I, H]; QMoE: uint8 packed */
  const void* fc1_scales;    /* QMoE only */
  const void* fc1_bias;      /* [E, I or 2I] */
  const void* fc2_weights;   /* [E, H, I] */
  const void* fc2_scales;
  const void* fc2_bias;      /* [E, H] */
  const void* fc3_weights;   /* [E, I, H] */
  const void* fc3_scales;
  const void* fc3_bias;      /* [E, I] */
  void* output;              /* [T, H] */
} moe_b200_tensors;

/* A tensor as the kernel context presents it (Ort::ConstValue analog). */
typedef struct moe_b200_tensor_ref {
  const void* data;   /* device pointer; NULL for an absent optional input */
  int32_t elem_type;  /* MOE_B200_* element type */
  int32_t rank;
  int64_t dims[4];
} moe_b200_tensor_ref;

typedef struct moe_b200_kernel moe_b200_kernel;
typedef struct moe_b200_prepacked moe_b200_prepacked;  /* QMoE weight prepack (below) */

/* ---------------------------------------------------------------- library */

int moe_b200_abi_version(void);

/* Message of the last non-OK status returned on this thread ("" if none). */
const char* moe_b200_last_error(void);

/* ------------------------------------------------------- operator kernels */

/* Creates the kernel object for one node.  op_type is "MoE" or "QMoE"; attributes
 * come as name/value strings with the schema's names and defaults.  Replaces the
 * create lambda of ONNX_OPERATOR_VERSIONED_KERNEL_EX (musa/ep/src/kernels/utils.h:160-207)
 * and OpKernelBase::CreateKernelImpl (kernels/shared_inc/kernel_base.h:36-43). */
int moe_b200_kernel_create(const char* op_type, int32_t num_attrs,
                           const char* const* attr_names,
                           const char* const* attr_values,
                           moe_b200_kernel** kernel);

/* Runs the node on `stream` (a cudaStream_t; NULL = legacy default stream).
 * inputs[] follows the schema's input order; absent optional inputs have
 * data == NULL.  The output tensor is caller-allocated with the input's shape.
 * Workspace comes from a per-kernel, per-stream cache (stream-ordered
 * allocation).  Replaces OpKernelBase::ComputeImpl (kernel_base.h:45-84). */
int moe_b200_kernel_compute(moe_b200_kernel* kernel, int32_t num_inputs,
                            const moe_b200_tensor_ref* inputs,
                            moe_b200_tensor_ref* output, void* stream);

/* Frees the kernel and its cached workspaces.  Replaces
 * OpKernelBase::ReleaseImpl (kernel_base.h:86-89). */
int moe_b200_kernel_release(moe_b200_kernel* kernel);

/* ------------------------------------------------ explicit-workspace path */

/* Bytes of device workspace that moe_b200_forward needs for this problem.
 * Replaces the scratch sizing before AllocateDeviceMemoryOnStream
 * (musa/ep/src/kernels/shared_inc/kernel_memory.h:241-252). */
int moe_b200_workspace_size(const moe_b200_problem* problem, size_t* bytes);

/* One MoE (expert_weight_bits == 0) or QMoE layer call on device pointers with a
 * caller-owned workspace (256-byte aligned, >= moe_b200_workspace_size).  Enqueues
 * work on `stream` only: no host synchronisation, no allocation. */
int moe_b200_forward(const moe_b200_problem* problem, const moe_b200_tensors* t,
                     void* workspace, size_t workspace_bytes, void* stream);

/* moe_b200_forward plus per-stage device times: stage_ms[0..6] receive the CUDA
 * event time of route, plan (scan + permutation), gather, QMoE dequantisation,
 * fc1(+fc3) GEMM, fc2 GEMM and combine, measured on `stream`.  Synchronises the
 * stream.  A measurement aid; it has no counterpart in the reference. */
int moe_b200_forward_timed(const moe_b200_problem* problem, const moe_b200_tensors* t,
                           void* workspace, size_t workspace_bytes, void* stream,
                           float* stage_ms, int32_t num_stages);

/* moe_b200_forward that also records the caller's CUDA events (cudaEvent_t handles,
 * num_events >= 8; NULL entries are skipped) on `stream` at the stage boundaries:
 * events[i] .. events[i+1] brackets stage i in the order of moe_b200_forward_timed.  No synchronisation, so back-to-back
 * calls keep the device busy and the stage times are those of a steady stream of calls.
 * A measurement aid; it has no counterpart in the reference. */
int moe_b200_forward_staged(const moe_b200_problem* problem, const moe_b200_tensors* t,
                            void* workspace, size_t workspace_bytes, void* stream,
                            void* const* events, int32_t num_events);

/* ---------------------------------------------------- expert parallelism */
/* Expert parallelism splits one layer over W ranks, rank r owning the experts
 * [r*E/W, (r+1)*E/W).  No counterpart in the reference (one EP drives one device,
 * musa/ep/src/ep_factory.cc:466-470); these three calls are the device side of the
 * exchange, the transport (an NCCL all-to-all) sits between them:
 *   1. moe_b200_ep_dispatch on every rank: route its T rows over all E experts and
 *      gather the T*k routed rows into send_rows in expert order, so the rows for rank
 *      r are the contiguous block [expert_offsets[r*E/W], expert_offsets[(r+1)*E/W]);
 *   2. exchange counts and rows; each rank runs moe_b200_expert_ffn on what it received
 *      (problem: its E/W experts, k = 1, num_rows = received rows; row_expert = local
 *      expert id of each row; router_probs unused; output row i = FFN of row i);
 *   3. send the FFN rows back in the same layout; moe_b200_ep_combine forms
 *      out[t] = sum_j w[t,j] * rows[permuted_pos[t,j]]. */
int moe_b200_ep_dispatch(const moe_b200_problem* problem, const void* router_probs,
                         const void* input, void* send_rows, int32_t* expert_offsets,
                         int32_t* permuted_pos, float* route_weight, void* workspace,
                         size_t workspace_bytes, void* stream);
int moe_b200_expert_ffn(const moe_b200_problem* problem, const moe_b200_tensors* t,
                        const int32_t* row_expert, void* workspace, size_t workspace_bytes,
                        void* stream);
int moe_b200_ep_combine(int32_t dtype, int64_t num_rows, int64_t hidden_size, int32_t k,
                        const void* expert_rows, const int32_t* permuted_pos,
                        const float* route_weight, void* output, void* stream);

/* ------------------------------------------------------ hot-path stages */

/* Router: softmax + top-k (+ renormalisation) of every row of router_probs
 * [T, E] (dtype FLOAT/FLOAT16/BFLOAT16).  expert_idx int32 [T, k],
 * route_weight float [T, k].  normalize_routing_weights: 0 = probabilities of the full
 * softmax, 1 = softmax over the k selected, 2 = sparse-mixer top-2 (k = 2: each pick's
 * weight is its softmax probability over the experts within 2 * 0.01 relative distance
 * of the pick's logit).  Analog of the reference's Softmax + TopK
 * (musa/ep/src/kernels/math/softmax_impl.mu:49, topk_impl.mu:46-65). */
int moe_b200_route(const void* router_probs, int32_t dtype, int64_t num_rows,
                   int64_t num_experts, int32_t k, int32_t normalize_routing_weights,
                   int32_t* expert_idx, float* route_weight, void* stream);

/* moe_b200_route without any device allocation, for callers that cannot allocate
 * where they route (memory planned up front, or owned by an arena that only hands
 * out inputs and outputs).  No counterpart in the reference.  Same arguments and
 * results as moe_b200_route; its scratch is a static 256 KiB device array, so
 * ceil(num_rows / 256) * num_experts must be <= 65536 (else INVALID_ARGUMENT).
 * All calls on a device share that array: calls overlapping on the GPU race.  The
 * first call on a device looks up the array's address; make it before any stream
 * capture. */
int moe_b200_route_noalloc(const void* router_probs, int32_t dtype, int64_t num_rows,
                           int64_t num_experts, int32_t k, int32_t normalize_routing_weights,
                           int32_t* expert_idx, float* route_weight, void* stream);

/* Dispatch plan for expert_idx [T, k]: expert_offsets int32 [E+1] (exclusive
 * scan of the counts), permuted_pos int32 [T*k] (position of routed row t*k+j)
 * and permuted_src int32 [T*k] (inverse).  Order: expert, then token, then slot.
 * `workspace` must hold moe_b200_permute_workspace_size() bytes. */
size_t moe_b200_permute_workspace_size(int64_t num_rows, int32_t k,
                                       int64_t num_experts);
int moe_b200_permute(const int32_t* expert_idx, int64_t num_rows, int32_t k,
                     int64_t num_experts, int32_t* expert_offsets,
                     int32_t* permuted_pos, int32_t* permuted_src,
                     void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------ runtime (CUDA retarget) */

typedef struct moe_b200_device_props {
  char name[256];
  uint32_t vendor_id;        /* 0x10DE */
  int32_t device_id;
  int32_t sm_count;
  int32_t cc_major, cc_minor;
  uint64_t total_memory;
  int32_t pci_bus_id;
} moe_b200_device_props;

/* Device discovery (musa/ep/src/ep_factory.cc:389-455). */
int moe_b200_device_count(int32_t* count);
int moe_b200_device_props_get(int32_t device_id, moe_b200_device_props* props);
int moe_b200_set_device(int32_t device_id);

/* Provider options of one session, parsed from the option key/value strings the
 * session carries (ParseMusaProviderOptionsFromSession + ValidateMusaProviderOptions,
 * musa/ep/src/ep_factory.cc:106-202, and the session entry
 * ep.musa.enable_prepack_weight_sharing read in CreateEpImpl, :472-478).  Keys:
 * device_id, has_user_compute_stream, user_compute_stream (a cudaStream_t address in
 * decimal or 0x-hex; "", "0" and "nullptr" mean none), use_ep_level_unified_stream,
 * do_copy_in_default_stream, ep.musa.enable_prepack_weight_sharing, and the
 * expert-parallel keys ep_world_size / ep_rank.  Unknown keys are ignored (they belong
 * to other providers).  Integers must be whole decimal strings; the flags must be 0 or
 * 1; device_id >= 0; a user stream implies has_user_compute_stream = 1 and
 * use_ep_level_unified_stream = 1.  Any violation returns INVALID_ARGUMENT naming the
 * option. */
typedef struct moe_b200_provider_options {
  int32_t device_id;                     /* default 0 */
  int32_t has_user_compute_stream;       /* default 0 */
  void* user_compute_stream;             /* default NULL */
  int32_t use_ep_level_unified_stream;   /* default 0 */
  int32_t do_copy_in_default_stream;     /* default 1 */
  int32_t enable_prepack_weight_sharing; /* default 0 */
  int32_t ep_world_size;                 /* default 1 */
  int32_t ep_rank;                       /* default 0 */
} moe_b200_provider_options;

int moe_b200_provider_options_parse(int32_t num_options, const char* const* keys,
                                    const char* const* values,
                                    moe_b200_provider_options* options);

/* Allocator (musa/ep/src/ep_allocator.h:86-321). */
int moe_b200_alloc(size_t bytes, void** ptr);
int moe_b200_free(void* ptr);
int moe_b200_alloc_pinned(size_t bytes, void** ptr);
int moe_b200_free_pinned(void* ptr);

/* Sync stream and notification (musa/ep/src/ep_stream.cc:30-185). */
int moe_b200_stream_create(void** stream);
int moe_b200_stream_destroy(void* stream);
int moe_b200_stream_synchronize(void* stream);
int moe_b200_notification_create(void** event);
int moe_b200_notification_activate(void* event, void* stream);   /* record */
int moe_b200_notification_wait(void* event, void* stream);       /* stream wait */
int moe_b200_notification_synchronize(void* event);              /* host wait */
int moe_b200_notification_destroy(void* event);

/* Data transfer (musa/ep/src/ep_data_transfer.cc:108-227).  kind: 0 = host to host,
 * 1 = H2D, 2 = D2H, 3 = D2D.  H2D and D2D are ordered on `stream` and return at once.
 * D2H returns with the data in place: it waits for `stream` only, or, when `stream` is
 * NULL, for the whole device before copying.  Host to host waits for `stream` (the
 * source's producer, if any) and copies on the host.  bytes == 0 or dst == src: no-op. */
int moe_b200_copy(void* dst, const void* src, size_t bytes, int32_t kind,
                  void* stream);

/* Pre-MoE rows in one pass: h = input (+ skip), stored as residual_out when skip is set;
 * normed = h * rsqrt(mean(h^2) + epsilon) * gamma (gamma fp32 [H]); router_logits [T, E]
 * = normed . router_weight[e] (router_weight [E, H], fp32 accumulation over the rounded
 * normed values).  The steps that produce an MoE node's input and router_probs in a
 * transformer block: the plugin's fused RMS normalisation
 * (musa/ep/src/fusion/rms_norm_fusion.cc:185, kernels/nn/rms_norm_impl.mu:10-45) and the
 * router MatMul (kernels/math/matmul.cc:239-332).  hidden_size % 8 == 0; buffers 16-byte
 * aligned; skip, residual_out and normed may be NULL. */
int moe_b200_norm_router(int32_t dtype, int64_t num_rows, int64_t hidden_size,
                         int64_t num_experts, const void* input, const void* skip,
                         const float* gamma, float epsilon, const void* router_weight,
                         void* residual_out, void* normed, void* router_logits, void* stream);

/* --------------------------------------- device-side expert parallelism (P2P) */

/* Expert-parallel layer over the GPUs of one node with no host synchronisation and no
 * collective library on the data path: rank r of W owns experts [r*E/W, (r+1)*E/W) and
 * one IPC-shared device region (receive buffer, return buffer, count matrix, flags).
 * Per call the ranks exchange per-expert counts with peer stores, the dispatch gather
 * writes routed rows into the owners' receive buffers, the fc2 epilogue writes the FFN
 * rows back into the senders' return buffers, and flags (bounded waits) order the steps.
 * The reference EP has no multi-device path (musa/ep/src/ep_factory.cc:466-470); these
 * entries are the dispatch / combine exchange of the MoE path.  fp16/bf16 MoE and fp16
 * QMoE (int4/int8 codes converted inside the tensor-core GEMM on the received rows). */
typedef struct moe_b200_ep_comm moe_b200_ep_comm;

/* Allocates this rank's region for calls of up to max_rows tokens with k <= k_max. */
int moe_b200_ep_comm_create(int32_t rank, int32_t world, int64_t max_rows, int32_t k_max,
                            int64_t hidden_size, int64_t num_experts, int32_t dtype,
                            moe_b200_ep_comm** comm);
/* Bytes of one rank's handle: its cudaIpcMemHandle_t followed by the arguments its
 * region was created with (rank, world, max_rows, k_max, hidden_size, num_experts, dtype). */
int moe_b200_ep_comm_handle_size(size_t* bytes);
int moe_b200_ep_comm_get_handle(moe_b200_ep_comm* comm, void* handle);
/* handles: world handles in rank order (this rank's own entry is ignored).  Every rank
 * must have created its communicator with the same world, max_rows, k_max, hidden_size,
 * num_experts and dtype, since peers write at offsets computed from their own layout:
 * any difference returns INVALID_ARGUMENT before a peer region is opened. */
int moe_b200_ep_comm_connect(moe_b200_ep_comm* comm, const void* handles);
/* Frees this rank's region: every rank must have finished its last moe_b200_ep_forward
 * (e.g. a barrier after a stream synchronisation) before any rank destroys its
 * communicator, since peers store into this region. */
int moe_b200_ep_comm_destroy(moe_b200_ep_comm* comm);
/* Workspace of one call (problem: this rank's num_rows, local num_experts = E / W). */
int moe_b200_ep_workspace_size(const moe_b200_ep_comm* comm,
                               const moe_b200_problem* problem, size_t* bytes);
/* One layer call on every rank of the communicator (all ranks call it the same number
 * of times).  t: this rank's input / router_probs [T, E] / output and its local weights
 * ([E/W, ...]).  A peer that does not take part makes the waits expire after 2 s with
 * device error code 6 in the workspace's error word. */
int moe_b200_ep_forward(moe_b200_ep_comm* comm, const moe_b200_problem* problem,
                        const moe_b200_tensors* t, void* workspace, size_t workspace_bytes,
                        void* stream);

/* moe_b200_ep_forward that also records the caller's CUDA events (num_events >= 9; NULL
 * entries skipped) on `stream` at the phase boundaries: events[i] .. events[i+1] brackets
 * route + plan, count exchange, row sends, wait for rows, fc1, fc2 with the return
 * stores, wait for the returned rows, combine.  A measurement aid; no counterpart in the
 * reference. */
int moe_b200_ep_forward_staged(moe_b200_ep_comm* comm, const moe_b200_problem* problem,
                               const moe_b200_tensors* t, void* workspace,
                               size_t workspace_bytes, void* stream, void* const* events,
                               int32_t num_events);

/* ------------------------------------------------ host-buffer call pipeline */

/* Calls of one layer on host-resident input, router logits and output (weights stay on
 * the device).  A session run with CPU inputs does this through the data transfer
 * (musa/ep/src/ep_data_transfer.cc:108-161) and, with do_copy_in_default_stream = 0,
 * separate copy streams ordered by notifications (musa/ep/src/ep_stream.cc:30-185):
 * here a copy-in stream, a compute stream and a copy-out stream with `depth` device
 * staging slots, so the copies of neighbouring calls overlap the compute of this one. */
typedef struct moe_b200_pipeline moe_b200_pipeline;

/* problem->num_rows is the largest call; `weights` holds the device weight/scale/bias
 * pointers (its input, router_probs and output are ignored); depth in [1, 8]. */
int moe_b200_pipeline_create(const moe_b200_problem* problem,
                             const moe_b200_tensors* weights, int32_t depth,
                             moe_b200_pipeline** pipeline);
/* Enqueues one call: H2D of host_input [num_rows, H] and host_router_probs
 * [num_rows, E], the layer, D2H into host_output [num_rows, H].  Never blocks the host;
 * the buffers must stay valid until moe_b200_pipeline_synchronize.  Pinned host memory
 * (moe_b200_alloc_pinned) lets the copies run asynchronously. */
int moe_b200_pipeline_submit(moe_b200_pipeline* pipeline, const void* host_input,
                             const void* host_router_probs, void* host_output,
                             int64_t num_rows);
/* Calls submitted from now on may take `prepacked` (moe_b200_prepack_create; NULL
 * detaches it); the pipeline holds its own reference. */
int moe_b200_pipeline_set_prepacked(moe_b200_pipeline* pipeline, moe_b200_prepacked* prepacked);
/* Waits for every submitted call (host outputs complete). */
int moe_b200_pipeline_synchronize(moe_b200_pipeline* pipeline);
int moe_b200_pipeline_destroy(moe_b200_pipeline* pipeline);

/* ------------------------------------------------------- QMoE weight prepack */

/* Dequantised copies of a QMoE node's expert weights, made once when the session is
 * initialised (the role of OpKernel::PrePack) and used by prefill-sized calls, which then
 * run the fp16/bf16 tensor-core GEMMs with no per-call dequantisation.  Decode-sized calls
 * keep streaming the packed codes, so the initializers stay needed (a plugin reports
 * is_packed = false).  share != 0 is the session option
 * "ep.musa.enable_prepack_weight_sharing" (parsed at musa/ep/src/ep_factory.cc:472-478):
 * nodes whose codes and scales have identical content, in any session of the process on
 * the same device, hold one reference-counted copy (matched by shape and a 64-bit content
 * hash). */
/* problem gives the weight shapes and attributes (num_rows is ignored); weights holds
 * the fc1/fc2(/fc3) codes and scales (other pointers are ignored).  Synchronises
 * `stream` before returning; the prepack may then be used from any stream. */
int moe_b200_prepack_create(const moe_b200_problem* problem, const moe_b200_tensors* weights,
                            int32_t share, void* stream, moe_b200_prepacked** prepacked);
/* Device bytes held and the current reference count (either pointer may be NULL). */
int moe_b200_prepack_info(const moe_b200_prepacked* prepacked, size_t* bytes, int32_t* refs);
/* Drops one reference; the memory is freed with the last one. */
int moe_b200_prepack_release(moe_b200_prepacked* prepacked);
/* moe_b200_workspace_size / moe_b200_forward for a call that may use `prepacked` (NULL
 * behaves as the plain entry points).  The call takes the prepacked weights when the
 * prepack matches the problem's shapes and the call is not decode-sized (and routes at
 * least MOE_B200_PREPACK_MIN_ROWS rows, num_rows * k, when that variable is set);
 * `t` must still hold the packed weights and scales, which other calls read. */
int moe_b200_workspace_size_prepacked(const moe_b200_problem* problem,
                                      const moe_b200_prepacked* prepacked, size_t* bytes);
/* `events`: NULL, or num_events >= 8 stage events recorded as by moe_b200_forward_staged. */
int moe_b200_forward_prepacked(const moe_b200_problem* problem, const moe_b200_tensors* t,
                               const moe_b200_prepacked* prepacked, void* workspace,
                               size_t workspace_bytes, void* stream, void* const* events,
                               int32_t num_events);
/* Kernel-object pre-pack: inputs[] in the QMoE schema order (input and router_probs may
 * be absent); the kernel keeps a reference and later computes whose weight inputs are the
 * same device pointers use it.  *is_packed is set to 0 (see above).  Call it before the
 * kernel's first compute, as ORT runs PrePack at session initialisation: it must not run
 * concurrently with a compute of the same kernel.  For an MoE kernel it packs nothing. */
int moe_b200_kernel_prepack(moe_b200_kernel* kernel, int32_t num_inputs,
                            const moe_b200_tensor_ref* inputs, int32_t share, void* stream,
                            int32_t* is_packed);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* MOE_B200_H_ */
