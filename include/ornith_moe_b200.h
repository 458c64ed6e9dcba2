/*
 * C ABI of the B200 routed mixture-of-experts layer (libornith_moe_b200.so).
 *
 * Drop-in for the routed library of ciru-ai/ornith-ciru-halo-agent
 * (libornith_routed_storage_n32.so, kernels/routed_storage/): the same symbol
 * names, argument order, layout struct and error behaviour, with CUDA types in
 * place of HIP ones.  The plugin binds them through ctypes exactly as
 * plugin-site/ornith_g256/native.py:45-85 and moe_shared.py:135-141 do.
 *
 * Fixed shapes: 256 routed experts, top-8, hidden H = 2048, intermediate
 * I = 512, quantisation group 256, Hadamard block 128.  Weight banks use the
 * reference's N32 storage (after plugin-site/ornith_g256/method.py:124-158):
 *   gate_codes  uint32 [256][32][8][32][32]   gate_meta  uint32 [256][32][8][32]
 *   down_codes  uint32 [256][64][2][32][32]   down_meta  uint32 [256][64][2][32]
 * Word j of group g for column n holds k = 256g + 8j + d in bits 4d..4d+3 (u4);
 * each metadata word is fp16 scale (low half) | fp16 offset (high half) and the
 * weight is scale*code + offset.
 *
 * Contract (routed_storage_n32_consumer.cpp:319-351 and the dense contract
 * kernels/dense_n32/dense_g256_api.h:32-44):
 *   - every launch is enqueued on `stream`; no allocation, no synchronisation,
 *     no host reads of device data (the expert-parallel buffer and IPC calls
 *     at the end are set-up functions outside this rule);
 *   - the caller owns every buffer; the workspace (size from get_layout) is not
 *     re-entrant: calls that share it must be ordered on one stream;
 *   - T == 0 returns success without touching any pointer; bad Tcap/T/bytes,
 *     null pointers or misaligned pointers return cudaErrorInvalidValue;
 *     launch failures return the CUDA error;
 *   - numerical faults are reported through sticky bits OR-ed into *flags_u32
 *     (never cleared by the library): 1 non-finite input/transform,
 *     2 invalid activation quantisation, 4 expert id outside [-1, 256),
 *     8 non-finite projection, 16 non-finite SiLU*up, 32 non-finite or
 *     overflowing output, 64 a bounded device wait gave up (results incomplete),
 *     128 (debug-bounds builds only) an index outside its buffer was redirected;
 *   - ids of -1 are padding and skip their slot.
 * Alignment: workspace 256 B; input, output, codes and metadata 16 B;
 * route weights, ids and flags 4 B.
 */
#ifndef ORNITH_MOE_B200_H
#define ORNITH_MOE_B200_H
#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORNITH_MOE_B200_EXPORT __attribute__((visibility("default")))

/* Same 15 size_t fields as OrnithRoutedDirectLayout
 * (kernels/routed_storage/routed_direct_api.h:11-14, native.py:16-20).
 * workspace_bytes is the size to allocate.  The other fields give the byte
 * offsets of this library's buffers (gate_low: int8 token activations,
 * gate_scales/gate_sums: their fp16 scales and int32 sums, middle: fp32
 * SiLU*up rows, down_low/down_scales/down_sums: quantised middle,
 * route_out: fp32 per-route down projections, final_f32: fp32 combined sum;
 * for T > 32 the rows of middle and route_out are in expert-slot order, see
 * ornith_moe_b200_gather_route_rows);
 * fields with no counterpart here (gate_x, gate_high, gate_y, down_x,
 * down_high) hold SIZE_MAX. */
typedef struct OrnithRoutedDirectLayout {
    size_t workspace_bytes, gate_x, gate_low, gate_high, gate_scales, gate_sums, gate_y;
    size_t middle, down_x, down_low, down_high, down_scales, down_sums, route_out, final_f32;
} OrnithRoutedDirectLayout;

/* Replaces ornith_routed_direct_get_layout (routed_storage_n32_consumer.cpp:309-318).
 * 0 <= Tcap <= 8192. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_routed_direct_get_layout(int Tcap, OrnithRoutedDirectLayout* out);

/* Replaces ornith_routed_direct_launch (routed_storage_n32_consumer.cpp:352-359,
 * routed_direct_api.h:15-18): A8 activations (int8, +-127) at both projections.
 * input bf16 [T,2048], route_weights fp32 [T,8], ids int32 [T,8] -> output bf16 [T,2048]. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_routed_direct_launch(
    const void* input_bf16, const void* route_weights_f32, const void* ids_i32,
    const void* gate_codes, const void* gate_meta, const void* down_codes, const void* down_meta,
    void* workspace, size_t bytes, void* output_bf16, void* flags_u32, int T, int Tcap, cudaStream_t stream);

/* Replaces ornith_routed_direct_launch_a4 (routed_storage_n32_consumer.cpp:360,
 * routed_direct_api.h:19-24): A4 activations (+-7) at both projections. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_routed_direct_launch_a4(
    const void* input_bf16, const void* route_weights_f32, const void* ids_i32,
    const void* gate_codes, const void* gate_meta, const void* down_codes, const void* down_meta,
    void* workspace, size_t bytes, void* output_bf16, void* flags_u32, int T, int Tcap, cudaStream_t stream);

/* Replaces ornith_routed_direct_launch_a4_prefill (routed_storage_n32_consumer.cpp:362-370):
 * A4 when T > 64, A8 otherwise. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_routed_direct_launch_a4_prefill(
    const void* input_bf16, const void* route_weights_f32, const void* ids_i32,
    const void* gate_codes, const void* gate_meta, const void* down_codes, const void* down_meta,
    void* workspace, size_t bytes, void* output_bf16, void* flags_u32, int T, int Tcap, cudaStream_t stream);

/* Replaces ornith_routed_storage_n32 (routed_storage_n32_consumer.cpp:372): returns 32,
 * the marker native.py:67-71 checks before using sole N32 storage. */
ORNITH_MOE_B200_EXPORT int ornith_routed_storage_n32(void);

/* Replaces ornith_routed_prefill_output_tile (routed_storage_n32_consumer.cpp:373):
 * 32, the production library's A4 prefill output tile.  Informational only. */
ORNITH_MOE_B200_EXPORT int ornith_routed_prefill_output_tile(void);

/* Replaces ornith_routed_shared_get_layout (routed_storage_n32_consumer.cpp:375-384).
 * 0 <= Tcap <= 16, as in the reference. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_routed_shared_get_layout(int Tcap, OrnithRoutedDirectLayout* out);

/* Replaces ornith_routed_direct_launch_shared_tables (routed_storage_n32_consumer.cpp:385-401):
 * the routed layer plus the shared expert as a ninth slot (A8).  Shared banks
 * have the routed layout with one expert.  shared_logit bf16 [T] (the shared
 * expert gate logit), shared_silu fp32 [65536] and shared_sigmoid bf16 [65536]
 * are the tables indexed by bf16 bits (native/shared_math_reference.safetensors).
 * Shared gate/up and down outputs are rounded to bf16; shared_output bf16 [T,2048]
 * = bf16(down * sigmoid[logit]) is written separately from output. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_routed_direct_launch_shared_tables(
    const void* input_bf16, const void* route_weights_f32, const void* ids_i32,
    const void* gate_codes, const void* gate_meta, const void* down_codes, const void* down_meta,
    const void* shared_gate_codes, const void* shared_gate_meta,
    const void* shared_down_codes, const void* shared_down_meta,
    const void* shared_logit, const void* shared_silu, const void* shared_sigmoid,
    void* workspace, size_t bytes, void* output_bf16, void* shared_output_bf16, void* flags_u32,
    int T, int Tcap, cudaStream_t stream);

/* ABI revision of this library (the counterpart of ornith_dense_g256_abi_version,
 * kernels/dense_n32/dense_g256_api.h:45).  Returns 1. */
ORNITH_MOE_B200_EXPORT uint32_t ornith_moe_b200_abi_version(void);

/* Number of kernels this library has enqueued since it was loaded (a host-side
 * counter, for benchmarks that report how many of this library's kernels ran
 * in a timed region).  No counterpart in the reference. */
ORNITH_MOE_B200_EXPORT unsigned long long ornith_moe_b200_kernel_launches(void);

/* Router top-8 with renormalised softmax weights, the role of vLLM's
 * fused_topk/topk_softmax (vllm/model_executor/layers/fused_moe/router/
 * fused_topk_router.py:69-102) for renormalize=True.  logits fp32 [T,256] ->
 * weights fp32 [T,8], ids int32 [T,8].  Slot order: descending logit, lower
 * expert index first on ties; weights = softmax over the eight selected logits
 * using the reference's portable exp.  Non-finite logits are never selected
 * (flag 1); unfilled slots get id -1 and weight 0.  0 <= T <= 8192. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_route_topk(
    const void* logits_f32, int T, void* weights_f32, void* ids_i32, void* flags_u32, cudaStream_t stream);

/* The MoE layer from router logits (the north-star operator: hidden states,
 * router logits, top-8, packed weights and scales in, combined hidden states
 * out).  Runs route_topk into the workspace, then the routed layer; when the
 * four shared banks are given it also runs the shared expert as a ninth slot
 * with logit = bf16(sum_k x[t,k]*shared_gate_weight[k]) in fp32 and writes
 * shared_output.  act_bits: 8 (A8), 4 (A4) or 0 (A4 when T > 64, else A8).
 * Shared-expert calls require act_bits 8 or 0 with T <= 64. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_launch_from_logits(
    const void* input_bf16, const void* logits_f32,
    const void* gate_codes, const void* gate_meta, const void* down_codes, const void* down_meta,
    const void* shared_gate_codes, const void* shared_gate_meta,
    const void* shared_down_codes, const void* shared_down_meta,
    const void* shared_gate_weight_bf16, const void* shared_silu, const void* shared_sigmoid,
    void* workspace, size_t bytes, void* output_bf16, void* shared_output_bf16, void* flags_u32,
    int T, int Tcap, int act_bits, cudaStream_t stream);

/* Slot-ordered weighted combine from explicit per-route rows: route_out fp32
 * [T*8][2048] (row 8t+s = slot s of token t), weights fp32 [T,8], ids int32
 * [T,8] -> output bf16 [T,2048] = bf16(sum over slots with a valid id, in slot
 * order from +0, of row*weight).  The arithmetic of reduce_slots
 * (routed_storage_n32_consumer.cpp:176-185); used by the expert-parallel home
 * rank after the per-slot rows come back from the expert owners.  Flag 32 on
 * non-finite or overflowing results. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_combine(
    const void* route_out_f32, const void* weights_f32, const void* ids_i32, int T,
    void* output_bf16, void* flags_u32, cudaStream_t stream);

/* The same combine from gathered rows: rows fp32 [n][2048] holds only the
 * per-slot rows that exist, and row_index int32 [T,8] gives the row of slot s
 * of token t (ignored where the id is -1 padding; an id outside -1..255, or
 * a valid id whose index is outside [0, n), raises flag 4 and contributes
 * nothing).  Saves the expert-
 * parallel home rank from scattering the returned rows into a dense
 * [T*8][2048] buffer.  No counterpart in the reference. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_combine_gathered(
    const void* rows_f32, int n_rows, const void* row_index_i32, const void* weights_f32, const void* ids_i32,
    int T, void* output_bf16, void* flags_u32, cudaStream_t stream);

/* Copies the fp32 down projections of n routes out of a workspace after a
 * layer call of T tokens on it (capacity Tcap): row i of rows fp32 [n][2048]
 * is the projection of route route_index[i] (8*token + slot, a slot with a
 * valid id).  The layer keeps these rows in route order for T <= 32 and in
 * expert-slot order on the tensor-core path, where this reads them through
 * its route -> row map.  A route index outside [0, 8T) raises flag 4 and
 * gives a zero row.  Used by the expert-parallel return exchange; no
 * counterpart in the reference. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_gather_route_rows(
    const void* workspace, size_t bytes, int T, int Tcap, const void* route_index_i32, int n, void* rows_f32,
    void* flags_u32, cudaStream_t stream);

/* Route-ordered copy of the same projections: rows fp32 [8T][2048] receives
 * row r for every route r with a valid id of the last layer call of T tokens
 * on the workspace; rows of padding slots hold unspecified values.  Used by the
 * expert-parallel exchange with fixed-size blocks; no counterpart in the
 * reference. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_scatter_route_rows(
    const void* workspace, size_t bytes, int T, int Tcap, void* rows_f32, cudaStream_t stream);

/* Dispatch plan of one expert-parallel layer call, in one launch: for T
 * tokens' ids int32 [T,8] and a placement (owner_i32 [256]: rank of each
 * expert, local_i32 [256]: its index in that rank's banks) over world ranks
 * (1..8), writes counts int64 [world][2] (tokens sent to each rank, (token,
 * slot) rows it returns), and for the n = sum of tokens sent: token_index
 * int64 [n] (grouped by destination, tokens ascending), dest int64 [n],
 * local_ids int32 [n][8] (the destination's bank numbering, -1 elsewhere),
 * slot_mask uint8 [n][8], and row_index int32 [T][8] (the row of each slot
 * among the rows that come back, -1 where no rank owns it).  The n-sized
 * buffers must hold T*world rows.  Ids -1 and outside 0..255 belong to no
 * rank.  T == 0 writes zero counts and touches nothing else.  No counterpart
 * in the reference, which runs one rank (plugin-site/ornith_g256/
 * moe_base.py:34-39). */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_ep_plan(
    const void* ids_i32, int T, const void* owner_i32, const void* local_i32, int world, void* counts_i64,
    void* token_index_i64, void* dest_i64, void* local_ids_i32, void* slot_mask_u8, void* row_index_i32,
    cudaStream_t stream);

/* Expert-parallel exchanges over NVLink peer memory.  Each rank owns a
 * receive buffer made by ep_buffer_alloc (zeroed device memory), shared with
 * the other ranks of the node through a CUDA IPC handle (ep_ipc_handle: 64
 * bytes; ep_ipc_open/_close on the peers); the caller lays out rows and flag
 * arrays inside it.  A flag array holds 2*world uint32 words: the epoch each
 * other rank raised, then that rank's status word (its flag-64 bit, stored
 * before the epoch), so that a rank whose own wait ran out makes every rank
 * it sends to report flag 64 too.  ep_return_p2p: after a layer call
 * of T tokens on `workspace`, rows [seg[h], seg[h+1]) of route_index (the
 * routes whose down projections go home to rank h; seg a host array of
 * world+1 entries) are copied to rows dst_offset[h]... of dst_rows[h] (host
 * arrays of world entries; entry `me` is this rank's own buffer), then
 * `epoch` is stored into slot `me` of every other rank's flag array
 * (signals[h]).  Every destination range must lie inside dst_capacity_rows,
 * which is checked before the launch.  counter_u32 is a zeroed device word
 * per stream.  ep_wait_signals: waits until every other rank's epoch in this
 * rank's array has reached `epoch`, for at most the peer wait limit (then
 * flag 64), and ORs their status bits into flags_u32.  Plain stores and loads
 * only (no TMA, no multicast).  No counterpart in the reference, which runs
 * one rank. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_ep_buffer_alloc(size_t bytes, void** ptr);
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_ep_buffer_free(void* ptr);
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_ep_ipc_handle(const void* base, void* handle_out);
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_ep_ipc_open(const void* handle, void** ptr);
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_ep_ipc_close(void* ptr);
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_ep_return_p2p(
    const void* workspace, size_t bytes, int T, int Tcap, const void* route_index_i32, int n, const int32_t* seg,
    void* const* dst_rows, const int64_t* dst_offset, int64_t dst_capacity_rows, void* const* signals, int world,
    int me, uint32_t epoch, void* counter_u32, void* flags_u32, cudaStream_t stream);
/* The dispatch direction: sent row i of a dispatch plan (token_index int64,
 * local_ids int32 [n][8], rows [seg[d], seg[d+1]) to expert rank d) is stored
 * as token row x[token_index[i]] (bf16 [T][2048]) and its ids at row
 * dst_offset[d] + i - seg[d] of expert rank d's buffers (dst_x, dst_ids), then
 * `epoch` goes into slot `me` of the other ranks' dispatch flag arrays. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_ep_dispatch_p2p(
    const void* x_bf16, int T, const void* token_index_i64, const void* local_ids_i32, int n, const int32_t* seg,
    void* const* dst_x, void* const* dst_ids, const int64_t* dst_offset, int64_t dst_capacity_rows,
    void* const* signals, int world, int me, uint32_t epoch, void* counter_u32, void* flags_u32,
    cudaStream_t stream);
/* The fixed-size exchange over peer memory (every rank T tokens; no host
 * value changes between calls, so a step can be captured in a CUDA graph).
 * Receive buffers come in two sets, used by calls of odd and even number; the
 * call number is a uint32 in device memory (epoch_u32, zero at first).
 * ep_fixed_dispatch: row me*T + t of every rank d's token buffer (dst_x, host
 * array [2][world], each set dst_capacity_rows >= world*T rows) receives x[t]
 * (bf16 [T][2048]) and its ids buffer (dst_ids) local_ids[d][t] (int32
 * [world][T][8]); then the call number goes into slot `me` of the others'
 * dispatch flags (with this rank's flag-64 bit from flags_u32 as its status
 * word) and into *epoch_u32.  ep_fixed_return: after the layer call on the
 * world*T received rows (ids int32 [world*T][8], capacity Tcap), each slot
 * with a valid local id of row h*T + t goes to row t*8 + s of home h's result
 * buffer (dst_rows, [2][world], each set dst_capacity_rows >= T*8 rows), then
 * the call number into the others' return flags.  Capacities too small for
 * those rows are refused before the launch.  ep_wait_epoch: waits, bounded
 * (flag 64), until every other rank's epoch reaches *epoch_u32, and ORs their
 * status bits into flags_u32. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_ep_fixed_dispatch(
    const void* x_bf16, const void* local_ids_i32, int T, void* const* dst_x, void* const* dst_ids,
    int64_t dst_capacity_rows, void* const* signals, int world, int me, void* epoch_u32, void* counter_u32,
    const void* flags_u32, cudaStream_t stream);
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_ep_fixed_return(
    const void* workspace, size_t bytes, int T, int Tcap, const void* ids_i32, void* const* dst_rows,
    int64_t dst_capacity_rows, void* const* signals, int world, int me, const void* epoch_u32, void* counter_u32,
    void* flags_u32, cudaStream_t stream);
/* The fixed exchange with the rank-partial combine.  ep_fixed_dispatch_weights:
 * ep_fixed_dispatch that also stores local_w[d][t] (fp32 [world][T][8], the
 * weights of rank d's slots, 0 elsewhere) into rank d's weight buffer
 * (dst_w, [2][world], each set world*T rows of 8).  ep_fixed_return_partial:
 * after the layer call on the world*T received rows with those weights, row
 * h*T + t of the layer's fp32 sums (the workspace's final_f32, this rank's
 * partial over its slots of token t of home rank h) goes to row me*T + t of
 * home h's partial buffer (dst_part, [2][world], each set dst_capacity_rows
 * >= world*T rows of 2048 fp32) when the token has a slot here, then the call
 * number into the others' return flags. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_ep_fixed_dispatch_weights(
    const void* x_bf16, const void* local_ids_i32, const void* local_w_f32, int T, void* const* dst_x,
    void* const* dst_ids, void* const* dst_w, int64_t dst_capacity_rows, void* const* signals, int world, int me,
    void* epoch_u32, void* counter_u32, const void* flags_u32, cudaStream_t stream);
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_ep_fixed_return_partial(
    const void* workspace, size_t bytes, int T, int Tcap, const void* ids_i32, void* const* dst_part,
    int64_t dst_capacity_rows, void* const* signals, int world, int me, const void* epoch_u32, void* counter_u32,
    void* flags_u32, cudaStream_t stream);
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_ep_wait_epoch(
    const void* signals_u32, int world, int me, const void* epoch_u32, void* flags_u32, cudaStream_t stream);
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_ep_wait_signals(
    const void* signals_u32, int world, int me, uint32_t epoch, void* flags_u32, cudaStream_t stream);
/* The limit of every wait on another rank (ep_wait_signals, ep_wait_epoch), in
 * nanoseconds of the GPU's global timer: 1 s by default, 1 us to 60 s
 * accepted (cudaErrorInvalidValue otherwise).  Process-wide; read when a wait
 * is launched, so a captured graph keeps the value of its capture.  Waits
 * inside one kernel on its own copies and CTAs keep a fixed 1 s limit.  No
 * counterpart in the reference. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_set_peer_wait_limit_ns(uint64_t limit_ns);
ORNITH_MOE_B200_EXPORT uint64_t ornith_moe_b200_peer_wait_limit_ns(void);

/* Router logits, the router linear ahead of the operator
 * (iu4_correctness/gates_projection.py:17-25): input bf16 [T,2048],
 * router_weight bf16 [256,2048] -> logits fp32 [T,256], each the fp32 sum
 * over k of f32(x)*f32(w).  The reference's reduction order is unspecified;
 * these agree with an exact sum to fp32 rounding. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_router_logits(
    const void* input_bf16, const void* router_weight_bf16, int T, void* logits_f32, cudaStream_t stream);

/* The router linear followed by ornith_moe_b200_launch_from_logits: the
 * logits are written to logits_f32 [T,256] (caller memory) and routed from
 * there.  Same workspace, outputs and flags as the from-logits entry.  At
 * T = 1 on the fused decode path one launch does both: the single-token
 * kernel computes the logits (the same bits as ornith_moe_b200_router_logits),
 * writes them to logits_f32 and routes from its own copy; where that kernel
 * does not fit the device the two launches run instead. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_launch_from_hidden(
    const void* input_bf16, const void* router_weight_bf16, void* logits_f32,
    const void* gate_codes, const void* gate_meta, const void* down_codes, const void* down_meta,
    const void* shared_gate_codes, const void* shared_gate_meta,
    const void* shared_down_codes, const void* shared_down_meta,
    const void* shared_gate_weight_bf16, const void* shared_silu, const void* shared_sigmoid,
    void* workspace, size_t bytes, void* output_bf16, void* shared_output_bf16, void* flags_u32,
    int T, int Tcap, int act_bits, cudaStream_t stream);

/* Workspace size for ornith_moe_b200_launch_from_logits (0 <= Tcap <= 8192). */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_get_layout(int Tcap, size_t* workspace_bytes);

/* ornith_routed_direct_launch (A8) for callers that cannot allocate device
 * memory: plugins inside frameworks that own every allocation and pass only
 * inputs and outputs, embedders without access to an allocator at the launch
 * site, and code that must not call cudaMalloc while others capture the
 * stream.  No counterpart in the reference.  The scratch is a fixed 1 MiB
 * array inside this library that every GPU loading the library keeps until
 * exit; it limits a call to T <= 8 tokens (larger T: cudaErrorInvalidValue).
 * Every call on a device shares that array, so calls that can overlap on the
 * GPU race: order them on one stream.  The first call on a device looks up the
 * array's address and should come before any stream capture; that address is
 * kept for the life of the process, so calls after cudaDeviceReset (or after
 * the device's primary context was destroyed and made again) are not
 * supported.  The library calls no allocator.  It always runs the fused decode
 * kernel: ORNITH_MOE_B200_PATH=generic and the NVTX layer range of the
 * workspace entry do not apply to it.  Arguments and results otherwise as
 * ornith_routed_direct_launch. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_routed_direct_launch_noalloc(
    const void* input_bf16, const void* route_weights_f32, const void* ids_i32,
    const void* gate_codes, const void* gate_meta, const void* down_codes, const void* down_meta,
    void* output_bf16, void* flags_u32, int T, cudaStream_t stream);

/* One-time repack of the reference checkpoint's N16 banks into N32 storage
 * (plugin-site/ornith_g256/method.py:124-158, prepare_n32_weights):
 * codes [E][N/16][K/256][32][16] -> [E][N/32][K/256][32][32], metadata
 * [E][N/16][K/256][16] -> [E][N/32][K/256][32].  N a multiple of 32, K of 256.
 * Source and destination must not overlap. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_moe_b200_repack_n16_to_n32(
    const void* codes_n16, const void* meta_n16, void* codes_n32, void* meta_n32,
    int experts, int N, int K, cudaStream_t stream);

/* ------------------------------------------------------------------------
 * Dense G256 projections (Ornith's dense layers): drop-in for the reference's
 * dense library (kernels/dense_n32/dense_g256_api.h, dense_g256_consumer.cpp),
 * same symbols, arguments and return codes.  Shapes: N a positive multiple of
 * 16, at most 12288 (or exactly 248320); K a positive multiple of 256, at most
 * 8192; 0 <= M <= Mcap <= 8192; bits 8; transform 128.
 * Banks: codes U32[N/16][K/256][32][16] (word j of group g for column n holds
 * k = 256g + 8j + d in bits 4d), metadata U32[N/16][K/256][16] = fp16 scale
 * (low half) | fp16 offset (high half); the N32 entry takes the N32 shadow
 * U32[N/32][K/256][32][32] / [N/32][K/256][32] (plugin-site/ornith_g256/
 * dense_n32.py:30-31).  Arithmetic: bf16 -> fp32, H128 x 0x3db504f3, A8 per
 * 256-group, exact integer dots, per column over ascending groups
 * value += w_scale*(sa*dot) + w_offset*(sa*sum) without FMA, bf16 RNE.
 * Flags (sticky, dense_g256_api.h:14-19): 1 non-finite transform input or
 * output, 2 invalid activation, 4 non-finite projection, 8 bf16 with an
 * all-ones exponent.  M == 0 returns success without touching a pointer
 * (the N32 entry rejects it, as the reference does).  Alignment: input 16 B
 * (the reference asks 2), workspace 256 B, codes, metadata and flags 4 B,
 * output 2 B; workspace, output and flags must not overlap any other buffer.
 * ------------------------------------------------------------------------ */

/* Same 7 size_t fields as the reference (dense_g256_api.h:11-13,
 * native.py:11-13).  Here `low` is the int8 activations [Mcap,K], `scales`
 * fp16 [Mcap,K/256], `sums` int32 [Mcap,K/256], `projection` the fp32
 * diagnostic [Mcap,N]; `transformed` and `high` hold SIZE_MAX. */
typedef struct OrnithDenseG256Layout {
    size_t workspace_bytes, transformed, low, high, scales, sums, projection;
} OrnithDenseG256Layout;

/* Replaces ornith_dense_g256_abi_version (dense_g256_api.h:45).  Returns 1. */
ORNITH_MOE_B200_EXPORT uint32_t ornith_dense_g256_abi_version(void);

/* Replaces ornith_dense_g256_get_layout (dense_g256_api.h:46,
 * dense_g256_consumer.cpp:162-171). */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_dense_g256_get_layout(int Mcap, int N, int K, int bits,
                                                                 OrnithDenseG256Layout* out);

/* Replaces ornith_dense_g256_launch (dense_g256_api.h:47-50,
 * dense_g256_consumer.cpp:172-190): input bf16 [M,K] -> output bf16 [M,N]
 * from an N16 bank.  geometry 0, 1 or 2 is accepted and gives identical
 * results (the reference's WMMA/compact job shapes). */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_dense_g256_launch(
    const void* input_bf16, const void* codes, const void* metadata,
    void* workspace, size_t workspace_bytes, void* output_bf16, void* flags_u32,
    int M, int Mcap, int N, int K, int bits, int transform, int geometry, cudaStream_t stream);

/* Replaces ornith_dense_g256_launch_n32 (dense_g256_consumer.cpp:360-379):
 * the same projection from the N32 shadow bank, 1 <= M <= 16, N a multiple
 * of 32, geometry 2. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_dense_g256_launch_n32(
    const void* input_bf16, const void* codes, const void* metadata,
    void* workspace, size_t workspace_bytes, void* output_bf16, void* flags_u32,
    int M, int Mcap, int N, int K, int bits, int transform, int geometry, cudaStream_t stream);

/* Replaces ornith_dense_g256_n32_rows (dense_g256_consumer.cpp:380): 16. */
ORNITH_MOE_B200_EXPORT int ornith_dense_g256_n32_rows(void);

/* Replaces ornith_dense_g256_prepare_bf16 (dense_g256_api.h:51-59,
 * dense_g256_consumer.cpp:231-247): transformed bf16 [M,K] = bf16(H128(x))
 * and weights bf16 [N,K] = bf16(scale*code + offset) from the N16 bank, for a
 * caller-side bf16 GEMM transformed @ weights^T (the reference's prefill path,
 * native.py:138-149).  No workspace.  Alignment 16 B for input, codes,
 * transformed and weights. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_dense_g256_prepare_bf16(
    const void* input_bf16, const void* codes, const void* metadata,
    void* transformed_bf16, void* weights_bf16, void* flags_u32, int M, int N, int K, cudaStream_t stream);

/* ------------------------------------------------------------------------
 * W8 LM head: drop-in for the reference's head library (kernels/head/
 * head_i8_tile_api.h, head_i8_tile_consumer.cpp), same symbols, arguments and
 * return codes.  K = 2048 in 16 groups of 128; N in {256, 1024, 4096, 65536,
 * 248320}; 0 <= M <= Mcap <= 64; geometry 0, 1 or 2 (identical results).
 * weights UINT32[N/16][K/16][4][16]: four signed int8 codes per word, lowest
 * k first (word kw of column n at ((n/16*128 + kw/4)*4 + kw%4)*16 + n%16);
 * scales fp16 [N][16], positive, >= 2^-14.  Per row: H128 per group, A8 per
 * 128-group, exact int32 dots, value += w_scale*(sa*dot) over ascending
 * groups without FMA, bf16 RNE.  Flags as the dense library (1, 2, 4, 8).
 * group_dots (optional, int32 [M][N][16]) receives the raw group dots;
 * null iff group_dots_bytes == 0.  Alignment: input 16 B (the reference asks
 * 2), workspace 256 B, weights, group_dots and flags 4 B, scales and output
 * 2 B; workspace, output, group_dots and flags overlap nothing.
 * ------------------------------------------------------------------------ */

/* Same 5 size_t fields as the reference (head_i8_tile_api.h:13-15,
 * native.py:23-25): activation_words UINT32[Mcap][512] in the reference's
 * format, activation_scales fp16 [Mcap][16], projection the fp32 diagnostic
 * [Mcap][N]; transformed holds SIZE_MAX. */
typedef struct OrnithHeadI8Layout {
    size_t workspace_bytes, transformed, activation_words, activation_scales, projection;
} OrnithHeadI8Layout;

/* Replaces ornith_head_i8_tile_abi_version (head_i8_tile_api.h:42).  Returns 1. */
ORNITH_MOE_B200_EXPORT uint32_t ornith_head_i8_tile_abi_version(void);

/* Replaces ornith_head_i8_tile_get_layout (head_i8_tile_api.h:43,
 * head_i8_tile_consumer.cpp:242-250). */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_head_i8_tile_get_layout(int Mcap, int N, OrnithHeadI8Layout* out);

/* Replaces ornith_head_i8_tile_launch (head_i8_tile_api.h:44-48,
 * head_i8_tile_consumer.cpp:251-291): input bf16 [M,2048] -> output bf16 [M,N]. */
ORNITH_MOE_B200_EXPORT cudaError_t ornith_head_i8_tile_launch(
    const void* input_bf16, const void* weights_i8, const void* scales_f16,
    void* workspace, size_t workspace_bytes, void* output_bf16,
    void* group_dots_i32, size_t group_dots_bytes, void* flags_u32,
    int M, int Mcap, int N, int geometry, cudaStream_t stream);

/* Replaces ornith_head_i8_tile_shortlist (head_i8_tile_consumer.cpp:293): 1. */
ORNITH_MOE_B200_EXPORT int ornith_head_i8_tile_shortlist(void);

#ifdef __cplusplus
}
#endif
#endif
