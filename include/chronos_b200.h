/* chronos_b200 — C ABI of the B200 (sm_100a) folded-expert MoE forward.
 *
 * Plain pointers and sizes only; every pointer inside `chronos_layer_t` and every buffer argument is a DEVICE
 * pointer owned by the caller (PyTorch in the shipped host layer).  The library allocates nothing, keeps no
 * global state besides immutable constant tables and a per-thread error string, launches on the stream it is
 * given and never synchronises, so the routed forward can be captured in a CUDA graph.  Every entry point
 * returns 0 on success and a negative `CHRONOS_E_*` code otherwise; `chronos_b200_last_error()` describes the
 * last failure of the calling thread.  Shape and alignment violations are rejected on the host before any
 * launch.  There is no CPU fallback.
 *
 * "Replaces" comments name the reference interface (path within the Chronos project : line) whose role the
 * entry point takes over.
 */
#ifndef CHRONOS_B200_H
#define CHRONOS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CHRONOS_OK 0
#define CHRONOS_E_SHAPE (-1)     /* a dimension violates the layout rules below               */
#define CHRONOS_E_ALIGN (-2)     /* a pointer is NULL or not 16-byte aligned                  */
#define CHRONOS_E_WORKSPACE (-3) /* workspace smaller than chronos_b200_workspace_bytes()     */
#define CHRONOS_E_LAUNCH (-4)    /* the CUDA runtime refused a launch (message has the cause) */
#define CHRONOS_E_ARG (-5)       /* an enum-like argument is out of range                     */

#define CHRONOS_DTYPE_F32 0
#define CHRONOS_DTYPE_BF16 1

#define CHRONOS_REGIME_AUTO 0   /* pick by pairs per slot */
#define CHRONOS_REGIME_STREAM 1 /* HBM-bound: packed banks streamed once, up to 8 pairs per pass */
#define CHRONOS_REGIME_TENSOR 2 /* dense: tcgen05 grouped GEMM, 128 pairs of one expert per tile */
#define CHRONOS_REGIME_STREAM_FP4 3 /* HBM-bound, banks fed as stored (e2m1 + ue4m3) to tcgen05 block-scaled FP4 MMA;
                                       needs the re-tiled bank copies (gu_t, dn_t); falls back to STREAM without them */
#define CHRONOS_REGIME_TENSOR_FP4 4 /* dense, block-scaled FP4 MMA with both operands streamed: 64 pairs of one expert x 3
                                       residual FP4 terms per tile; needs the re-tiled banks and v_dn, else falls back to
                                       CHRONOS_REGIME_TENSOR */

#define CHRONOS_ROUTER_SOFTMAX_TOPK 0 /* chronos_1t/models/vllm_chronos_moe.py:310-314     */
#define CHRONOS_ROUTER_SIGMOID_NOAUX 1 /* chronos_1t/models/glm53_chronos_moe.py:392-399    */
#define CHRONOS_ROUTER_SQRT_SOFTPLUS 2 /* chronos_1t/models/dsv41_chronos_moe.py:3402-3410: choose by
                                          sqrt(softplus(logit)) + bias, weigh by the unbiased scores, renorm, scaling */

/* One folded MoE layer resident in HBM.
 *
 * Dimensions: hidden H and inter I are multiples of 128 and at most 32768; n_experts = n_slots * group_size;
 * expert e lives in slot e / group_size as member e % group_size (chronos_1t/models/glm5_chronos_moe.py:439-440).
 * rank r is 16, 32, 64 or 128.  top_k <= 32.
 *
 * Banks and healers hold the on-disk bytes of the converter unchanged (suffix names from
 * chronos_1t/models/glm53_holo.py:45-51), stacked over slots / experts:
 *   gu_w   u8   [n_slots, 2I, H/2]   "s_gu.weight"      e2m1 nibbles, even column in the low nibble
 *   gu_s   e4m3 [n_slots, 2I, H/16]  "s_gu.weight_scale"
 *   gu_s2  f32  [n_slots]            "s_gu.weight_scale_2"
 *   gu_beta f32 [n_experts]          "s_gu.beta"
 *   dn_*   the same for "s_down.*" with shape [H, I/2] / [H, I/16]
 *   u_gu   e4m3 [n_experts, 2I, r]   "healer.u_gu"
 *   v_gu   e4m3 [n_experts, r, H]    "healer.v_gu"
 *   u_dn   e4m3 [n_experts, H, r]    "healer.u_down"
 *   v_dn_t e4m3 [n_experts, I, r]    "healer.v_down" TRANSPOSED once at load (on disk it is [r, I])
 *
 * Key tables are built on the host at load time from torch's CPU generator exactly as
 * chronos_1t/models/glm53_holo.py:66-86 draws them, then compacted:
 *   *_cin  u16 [n_experts, cols]     bits 0-14 = c_perm[j], bit 15 = (c_s1[c_perm[j]] < 0)
 *   *_cs2  u32 [n_experts, cols/32]  bit j%32 of word j/32 = (c_s2[j] < 0)
 *   *_rout u16 [n_experts, rows]     bits 0-14 = r_inv[i],  bit 15 = (r_s1[i] < 0)
 *   *_rs2  u32 [n_experts, rows/32]  bit = (r_s2[i] < 0)
 * with (rows, cols) = (2I, H) for gu and (H, I) for down.
 *
 * Optional always-on shared expert in plain (unfolded) NVFP4, the hub-expert format of
 * chronos_1t/models/vllm_chronos_moe.py:131-141: sh_gu_* [2*shared_inter, H/2|H/16], sh_dn_* [H, shared_inter/2|/16];
 * sh_gu_s2 f32 [2] = (gate_proj, up_proj) weight_scale_2, sh_dn_s2 f32 [1].
 * shared_inter == 0 disables it.  shared_inter must equal inter when non-zero.
 *
 * Optional (NULL when absent; needs H and I multiples of 256): the same bank bytes re-tiled once at load into the
 * operand images of the block-scaled FP4 tensor-core path - per (slot, 128-row block, 256-column stage) 16384 bytes
 * of nibbles in K-major core-matrix order followed by four 512-byte scale blocks (see chronos_b200_fp4_mma_probe):
 *   gu_t u8 [n_slots, 2I/128, H/256, 18432], dn_t u8 [n_slots, H/128, I/256, 18432], sh_gu_t / sh_dn_t without the
 *   slot axis.  A pure permutation of the "s_gu.weight" + "s_gu.weight_scale" bytes; the file format is untouched.
 * Optional: the shared expert in the STOCK 128 x 128 block-FP8 checkpoint format instead (the format the reference keeps it in,
 *   chronos_1t/models/glm53_chronos_moe.py:170-181): sh8_gu_w e4m3 [2*shared_inter, H] (gate rows, then up rows),
 *   sh8_gu_s f32 [2*shared_inter/128, H/128] "weight_scale_inv", sh8_dn_w e4m3 [H, shared_inter], sh8_dn_s f32
 *   [H/128, shared_inter/128]; value = float(e4m3) * scale_inv[row/128, col/128] (chronos_1t/models/glm53_tiers.py:74-95).
 *   With sh8_gu_w set the NVFP4 shared-expert pointers (sh_*) are ignored.
 * Optional tail lattice (tail_bits != 0; chronos_1t/models/chronos_moe_block.py:122-229, applied at
 *   chronos_1t/models/glm53_holo.py:362-366): per expert a matrix in natural weight space added to the reconstruction,
 *   tail_gu_p u8 [n_experts, 2I, H*bits/8] "tail.gu_packed", tail_gu_s e4m3 [n_experts, 2I, H/32 (2-bit) | H/64 (1-bit)]
 *   "tail.gu_scale", tail_dn_* the same with [H, I*bits/8] and [H, I/32 | I/64].  2-bit codes (4 per byte, column 4j in
 *   bits 0-1) index the Lloyd-Max levels (-1.510417, -0.452780, 0.452780, 1.510417); 1-bit codes (8 per byte, column 8j
 *   in bit 0) mean -1 / +1; the value is level * float(block scale).  With tail_bits set every entry point adds the term.
 * Optional: v_dn e4m3 [n_experts, r, I], "healer.v_down" exactly as on disk (kept beside its transposed copy); with it
 *   large batches run their healer products on the tensor cores.
 * Optional (rank 16 ... 64, with gu_t / dn_t): ut_gu f16 [n_experts, 2I/128, r/8, 128, 8] and ut_dn f16 [n_experts, H/128,
 *   r/8, 128, 8] - healer.u_gu / healer.u_down carried once at load into the row order and basis of the bank-pass
 *   accumulators (rows gathered by r_inv with the r_s1 sign and 1/beta, 128-row Walsh-Hadamard blocks, r_s2 sign), stored as
 *   K-major fp16 operand tiles of 128 rows, divided by the slot's scale_2 and by a power of two ut_scale f32 [2] = (gate_up,
 *   down) that keeps them in fp16 range (the kernel multiplies the other operand by it). With them the FP4 tensor regime adds the low-rank correction inside the bank
 *   pass (one more tensor-core step per tile into the same accumulators) instead of in a pass of its own that re-reads
 *   healer.u_* once per 8 pairs.
 */
typedef struct chronos_layer {
    int32_t hidden, inter, n_experts, group_size, n_slots, rank, top_k;
    int32_t router_kind;   /* CHRONOS_ROUTER_* */
    int32_t renorm;        /* sigmoid router: divide weights by their sum (norm_topk_prob) */
    float routed_scaling;  /* sigmoid router: routed_scaling_factor */
    int32_t shared_inter;
    int32_t tail_bits;     /* 0 = no tail; else gate_up bits (1 or 2) | down bits << 8 */
    const float* router_w; /* [n_experts, H] */
    const float* e_bias;   /* [n_experts] or NULL (sigmoid router's e_score_correction_bias) */
    const uint8_t* gu_w; const uint8_t* gu_s; const float* gu_s2; const float* gu_beta;
    const uint8_t* dn_w; const uint8_t* dn_s; const float* dn_s2; const float* dn_beta;
    const uint8_t* u_gu; const uint8_t* v_gu; const uint8_t* u_dn; const uint8_t* v_dn_t;
    const uint16_t* gu_cin; const uint32_t* gu_cs2; const uint16_t* gu_rout; const uint32_t* gu_rs2;
    const uint16_t* dn_cin; const uint32_t* dn_cs2; const uint16_t* dn_rout; const uint32_t* dn_rs2;
    const uint8_t* sh_gu_w; const uint8_t* sh_gu_s; const float* sh_gu_s2;
    const uint8_t* sh_dn_w; const uint8_t* sh_dn_s; const float* sh_dn_s2;
    const uint8_t* gu_t; const uint8_t* dn_t; const uint8_t* sh_gu_t; const uint8_t* sh_dn_t;
    const uint8_t* v_dn;
    const uint8_t* tail_gu_p; const uint8_t* tail_gu_s; const uint8_t* tail_dn_p; const uint8_t* tail_dn_s;
    const uint8_t* sh8_gu_w; const float* sh8_gu_s; const uint8_t* sh8_dn_w; const float* sh8_dn_s;
    const void* ut_gu; const void* ut_dn; const float* ut_scale;
} chronos_layer_t;

/* NVFP4 dequantisation probe: out[rows, cols] f32 = lut[nibble] * (float(e4m3 scale) * scale_2), evaluated
 * in fp32 in exactly that order (bit-exact target).
 * Replaces: unpack_nvfp4, chronos_1t/converter/convert_glm53_flash_colab.py:81-89
 *           (= chronos_1t/models/chronos_moe_block.py:109-119 with dtype=float32). */
int chronos_b200_dequant_nvfp4(const uint8_t* packed, const uint8_t* scale, const float* scale_2, float* out,
                               int rows, int cols, void* stream);

/* Block-FP8 dequantisation probe: out[rows, cols] f32 = float(e4m3 w[r, c]) * scale_inv[r / 128, c / 128] in fp32 (bit-exact
 * target); scale_inv f32 [ceil(rows/128), ceil(cols/128)].
 * Replaces: dequant_fp8_block(dtype=float32), chronos_1t/models/glm53_tiers.py:74-95. */
int chronos_b200_dequant_fp8_block(const uint8_t* w, const float* scale_inv, float* out, int rows, int cols, void* stream);

/* Weight-space reconstruction probe of ONE expert: out f32 = beta * unbind(bank) + U.V, plus the tail-lattice term
 * when the layer carries one (tail_bits != 0).  which = 0: gate_up [2I, H]; which = 1: down [H, I].  `scratch` holds
 * rows*cols floats.  Stream-ordered like every other entry point: no copy to the host, no synchronisation.
 * Replaces: reconstruct_group_experts(include_tail = tail_bits != 0), chronos_1t/models/glm53_holo.py:336-368. */
int chronos_b200_unfold_expert_fp32(const chronos_layer_t* layer, int expert, int which, float* out, float* scratch,
                                    void* stream);

/* The same reconstruction probe for callers that cannot provide scratch memory because they cannot allocate any:
 * code running inside a serving process whose framework has already claimed the GPU's memory for its own pool
 * (an extra cudaMalloc there can fail or fragment the pool), or code that must not call the allocator at this point
 * at all (a latency-critical step, a region where allocation calls are forbidden).  The row-axis intermediate is
 * kept in a 16 MiB array that is part of the library image on every GPU that loads it, so only matrices with
 * rows * cols <= 4,194,304 are accepted (e.g. 1536 x 2048); larger ones are refused with CHRONOS_E_SHAPE and a
 * message naming the limit - use the entry point above for those.  The entry point calls no cudaMalloc / cudaFree
 * and no allocating library routine.  The first call on a device looks up the array's device address (the device
 * must be current; that look-up is a runtime query, so make the first call on a device before any stream capture).  All calls on a device share the one array:
 * its previous contents are simply overwritten (nothing needs clearing), and two calls that overlap on the GPU -
 * different streams, or a second call issued before the first finished on another stream - race on it.
 * This entry point has no counterpart in the reference. */
int chronos_b200_unfold_expert_fp32_static(const chronos_layer_t* layer, int expert, int which, float* out, void* stream);

/* Router: fp32 logits in the fixed summation order (lane l of 32 sums k = 128 j + 4 l + i, j ascending then i = 0..3,
 * with FMAs from +0, then the xor butterfly 16,8,4,2,1), top-k descending with ties to the lower index, gate weights
 * per router_kind.
 * ids i32 [n_tokens, top_k], gates f32 [n_tokens, top_k], logits f32 [n_tokens, n_experts] (scratch, also returned).
 * Reads only hidden, n_experts, top_k, router_kind, renorm, routed_scaling, router_w and e_bias of `layer`, so an
 * expert-parallel shard can pass a description whose n_experts is the width of the full router table.
 * Replaces: the router blocks at chronos_1t/models/vllm_chronos_moe.py:310-314 and
 *           chronos_1t/models/glm53_chronos_moe.py:392-399. */
int chronos_b200_router_topk(const chronos_layer_t* layer, const void* x, int x_dtype, int n_tokens, int32_t* ids,
                             float* gates, float* logits, void* stream);

/* Router with the batch-coalesced selection policy for speculative verify batches: tokens come in streams of
 * tokens_per_stream (token 0 = the verified anchor, the rest drafts).  The anchor gets its natural top-k.  A draft keeps
 * its `keep` best natural experts, and fills the other top_k - keep places from its own natural top-`pool` candidates
 * ranked by choice score + `bonus` for experts the anchor selected too (ties to the better natural rank), so that fewer
 * distinct banks are streamed per step; it is never routed outside its natural top-`pool`.  pool == top_k or bonus == 0
 * reproduces chronos_b200_router_topk.  Gate weights follow router_kind on the unbiased scores of the picked experts.
 * Feed ids / gates to chronos_b200_folded_moe_routed.
 * Stands in for `_chronos_fused_topk_sigmoid_kernel`, which the reference only describes (README.md:56, :208, :372;
 * docs/CHRONOS_ARCHITECTURE_PAPER.md:270-277): its source is not part of the reference, so this is a clean-room policy
 * built to the stated invariants, not a transcription. */
int chronos_b200_router_topk_coalesced(const chronos_layer_t* layer, const void* x, int x_dtype, int n_tokens, int tokens_per_stream,
                                       int pool, int keep, float bonus, int32_t* ids, float* gates, float* logits, void* stream);

/* Bytes of caller-owned scratch the forward entry points need for n_tokens tokens (0 on bad arguments). */
size_t chronos_b200_workspace_bytes(const chronos_layer_t* layer, int n_tokens);

/* Whole layer, streaming regime (HBM-bound; any n_tokens, meant for decode-shaped batches):
 * y[n_tokens, H] = sum_k gate_k * Expert_{id_k}(x) (+ shared expert), router included.  Each distinct slot's
 * bank is read from HBM once per call for up to 8 (token, expert) pairs that hit it.  Uses the block-scaled FP4
 * tensor-core pass (CHRONOS_REGIME_STREAM_FP4) when the layer carries re-tiled banks and the workspace was laid
 * out for it (n_tokens * top_k < 16 * n_slots), otherwise the CUDA-core conversion pass (CHRONOS_REGIME_STREAM).
 * Replaces: ChronosGlm53SparseMoeBlock.forward_impl, chronos_1t/models/glm53_chronos_moe.py:474-483, with the
 *           experts evaluated as ChronosGlm5HolographicExpertGroup.forward_cold_fast does
 *           (chronos_1t/models/glm5_chronos_moe.py:149-195). */
int chronos_b200_folded_moe_decode(const chronos_layer_t* layer, const void* x, int x_dtype, int n_tokens, void* y,
                                   int y_dtype, void* workspace, size_t workspace_bytes, void* stream);

/* Whole layer, tensor-core regime (prefill-shaped batches): same result contract as folded_moe_decode; the two bank
 * passes run as grouped GEMMs on the 5th-generation tensor cores (tcgen05.mma, accumulators in tensor memory), with
 * the NVFP4 bank tiles converted to fp16 operands on the fly (exactly) and the scale_2 / r_s2 / Walsh-Hadamard step
 * fused into the epilogue.
 * Replaces: the grouped dense path of ChronosGlm53SparseMoeBlock.routed_forward,
 *           chronos_1t/models/glm53_chronos_moe.py:452-472. */
int chronos_b200_folded_moe_prefill(const chronos_layer_t* layer, const void* x, int x_dtype, int n_tokens, void* y,
                                    int y_dtype, void* workspace, size_t workspace_bytes, void* stream);

/* Whole layer with the regime chosen from the batch shape (tensor regime once n_tokens * top_k >= 16 * n_slots).
 * Replaces: ChronosGlm53SparseMoeBlock.forward, chronos_1t/models/glm53_chronos_moe.py:485-486 (which picks between
 *           its GEMV and grouped dense paths by pair count, :445). */
int chronos_b200_folded_moe_forward(const chronos_layer_t* layer, const void* x, int x_dtype, int n_tokens, void* y,
                                    int y_dtype, void* workspace, size_t workspace_bytes, void* stream);

/* Same, with routing supplied by the caller (ids < 0 are skipped; used by the expert-parallel host layer where
 * a rank only owns some slots).  ids i32 [n_tokens, top_k], gates f32 [n_tokens, top_k].  Tokens shared_first ..
 * shared_first + shared_count - 1 also get the shared expert's output added (0, n_tokens = all; count 0 = none; an
 * expert-parallel rank passes the block of tokens it is the home of).  regime is a CHRONOS_REGIME_* value.
 * Replaces: ChronosGlm53SparseMoeBlock.routed_forward, chronos_1t/models/glm53_chronos_moe.py:441-472. */
int chronos_b200_folded_moe_routed(const chronos_layer_t* layer, const void* x, int x_dtype, int n_tokens,
                                   const int32_t* ids, const float* gates, int shared_first, int shared_count, int regime,
                                   void* y, int y_dtype, void* workspace, size_t workspace_bytes, void* stream);

/* h[n_tokens, H] += y (when y != NULL); x_norm = h * rsqrt(mean(h^2) + eps) * (weight or 1), fp32 math.
 * Replaces: rms_norm + residual wiring, chronos_1t/models/glm53_engine.py:71-73 and :200-204. */
int chronos_b200_residual_rmsnorm(void* h, const void* y, const float* weight, void* x_norm, int dtype, int n_tokens,
                                  int hidden, float eps, void* stream);

/* Expert-parallel dispatch, device side (one process per GPU; experts sharded by slot, rank d owns experts
 * [d * experts_per_rank, (d + 1) * experts_per_rank)).  Fills, for every destination rank d, a fixed-capacity block:
 *   send_rows [world, capacity, hidden]  (x's dtype) the hidden rows of the local tokens that route >= 1 expert to d, each
 *             token ONCE per destination, in token order;
 *   send_meta i32 [world, capacity + 1, 2 * top_k + 2]: row p < capacity = (source token, top_k expert ids local to d or
 *             -1, top_k gates as fp32 bits, pad); row `capacity`, word 0 = rows used in the block;
 *   slot_of  i32 [n_tokens, world]: position of token t in d's block, or -1.
 * ids are GLOBAL expert ids [n_tokens, top_k] (< 0 skipped), gates f32.  A token that does not fit (more than
 * `capacity` tokens for one destination) is left out and *overflow (device int32, caller-cleared) is raised: the
 * caller checks it at the end of the step and repeats the step with capacity = n_tokens, which always fits.
 * The blocks are then exchanged by a collective with equal splits (NCCL all-to-all in the shipped host layer).
 * block_rows / meta_block_ints: distance between the blocks of consecutive destinations in send_rows (in rows) and in
 * send_meta (in 32-bit words); 0 = dense (capacity rows, (capacity + 1) * (2 top_k + 2) words).  With larger strides both can
 * live in ONE buffer - block d = capacity rows followed by the block's metadata - so one collective moves them.
 * No counterpart in the reference (single device; chronos_1t/docs/CHRONOS_ARCHITECTURE_PAPER.md:244 only names the idea). */
int chronos_b200_ep_pack(const void* x, int x_dtype, const int32_t* ids, const float* gates, int n_tokens, int top_k, int hidden,
                         int world, int experts_per_rank, int capacity, void* send_rows, int32_t* send_meta, int32_t* slot_of,
                         int32_t* overflow, int block_rows, long meta_block_ints, void* stream);

/* Received metadata blocks [world, capacity + 1, 2 * top_k + 2] (meta_block_ints words apart; 0 = dense) -> the routing
 * lists of the received rows: ids_out i32 [world * block_rows + tail_rows, top_k] (local expert ids; -1 for unused rows and
 * entries, for the rows capacity .. block_rows - 1 of every block and for the tail_rows rows at the end), gates_out f32
 * likewise; block_rows 0 = capacity.  No counterpart in the reference. */
int chronos_b200_ep_unpack_meta(const int32_t* recv_meta, int world, int capacity, int top_k, int32_t* ids_out, float* gates_out,
                                int block_rows, long meta_block_ints, int tail_rows, void* stream);

/* Expert-parallel combine on the home rank: y[t] = extra[t] + sum over ranks d = 0 .. world - 1 (in that order) of
 * back_rows[d, slot_of[t, d]] where slot_of >= 0.  back_rows [world, block_rows, hidden] (block_rows 0 = capacity) are the
 * partial-sum rows the peers returned (bf16 or f32), extra [n_tokens, hidden] (same dtype, or NULL) e.g. the shared expert's rows.
 * No counterpart in the reference. */
int chronos_b200_ep_combine(const void* back_rows, int dtype, const int32_t* slot_of, const void* extra, int n_tokens, int hidden,
                            int world, int capacity, void* y, int y_dtype, int block_rows, void* stream);

/* The same exchange by peer stores instead of a collective (ranks of one NVLink box whose receive buffers are mapped into
 * each other's address space, e.g. torch symmetric memory).  A receive buffer is world blocks of block_rows rows of hidden
 * elements; block s holds what rank s sent: capacity rows, then the block's metadata ((capacity + 1) x (2 top_k + 2) int32 as
 * in chronos_b200_ep_pack) starting at row `capacity`.
 *   chronos_b200_ep_pack_peer       fills block `my_rank` of EVERY rank's buffer: peer_bases = device array of world base
 *                                   pointers (entry d = rank d's buffer as mapped here; entry my_rank = the local buffer);
 *                                   also copies x behind the world blocks of the local buffer (n_tokens more rows).
 *   chronos_b200_ep_send_back_peer  copies block s of part_rows [world, block_rows, hidden] (as many rows as the count word of
 *                                   the metadata received from rank s, read at recv_base) into block `my_rank` of peer_back[s].
 *   chronos_b200_ep_barrier         pads = device array of world pointers to a few peer-writable 32-bit words per rank (word s
 *                                   of rank d's pad = last epoch rank s finished).  Tells every peer that this rank's stores
 *                                   issued before it on the stream are done and waits for the same from every peer; epoch must
 *                                   grow by one per call on every rank (wrap-around is fine).  The wait is bounded (about a
 *                                   second); on expiry CHRONOS_STATUS_EP_BARRIER is raised in *status (device int32) and the
 *                                   kernel returns - the caller must read it before it trusts the step.
 * Plain peer loads and stores only.  No counterpart in the reference. */
int chronos_b200_ep_pack_peer(const void* x, int x_dtype, const int32_t* ids, const float* gates, int n_tokens, int top_k, int hidden,
                              int world, int experts_per_rank, int capacity, void* const* peer_bases, int my_rank, int block_rows,
                              int32_t* slot_of, int32_t* overflow, void* stream);
int chronos_b200_ep_send_back_peer(const void* part_rows, int dtype, int hidden, int world, int block_rows, int capacity, int top_k,
                                   const void* recv_base, void* const* peer_back, int my_rank, void* stream);
int chronos_b200_ep_barrier(void* const* pads, int my_rank, int world, uint32_t epoch, int32_t* status, void* stream);

/* Operand-format probe of the block-scaled FP4 tensor-core path (tcgen05.mma kind::mxf4nvf4, e2m1 operands with a
 * ue4m3 scale per 16 elements): d_out f32 [128, b_rows] = (A * scaleA) (B * scaleB)^T over n_stages * 256 columns;
 * b_rows a multiple of 16 in 16..256 (32 = streaming regime, 192 = tensor regime).
 * a_image: n_stages x 18432 bytes, b_image: n_stages x (b_rows * 128 + 2048 * ceil(b_rows / 128)) bytes; per stage the
 * packed nibbles of a 128-row (resp. b_rows-row) x 256-column tile in K-major core-matrix order - byte(r, c, b) at
 * c * rows * 16 + r * 16 + b, c = 16-byte chunk along K - followed, per 64 columns, by one 512-byte scale block per
 * 128 rows (byte(r, s) of a block at (r % 32) * 16 + ((r % 128) / 32) * 4 + s).
 * status: one int32 the kernel raises bits in if a bounded wait expires (clear it first).
 * The values are what unpack_nvfp4 (chronos_1t/converter/convert_glm53_flash_colab.py:81-89) gives with
 * weight_scale_2 = 1; the reference has no tensor-core path to compare with beyond that. */
int chronos_b200_fp4_mma_probe(const uint8_t* a_image, const uint8_t* b_image, int n_stages, int b_rows, float* d_out,
                               int32_t* status, void* stream);

/* Profiling aid for the calling thread: with n_events = 8 CUDA events (cudaEvent_t handles, timing enabled) the
 * forward entry points record events[i] on the call's stream at their stage boundaries:
 *   0 start | 1 after router (2 launches) | 2 after plan | 3 after gate_up input transform | 4 after gate_up bank pass
 *   | 5 after SwiGLU / down input transform | 6 after down bank pass | 7 after combine.
 * (folded_moe_routed starts at boundary 1.)  n_events = 0 switches it off.  Events are not recorded otherwise.
 * No counterpart in the reference (it times whole calls with torch.cuda.Event,
 * benchmarks/dgx_spark_gb10_experiments.py:70-71). */
int chronos_b200_set_stage_events(void** events, int n_events);

/* Byte offset, inside a workspace laid out for n_tokens, of the int32 device status word that the forward entry
 * points clear at the start of a call and kernels raise on a device-side anomaly.  Every wait inside a kernel (on a
 * shared-memory barrier, or on the other CTAs of its grid) is bounded to about a second; a kernel whose wait runs
 * out raises its bit, stops feeding its pipeline, lets its copies in flight land, frees its tensor memory and
 * returns - the output of that call is then garbage, the context stays usable.  Bits:
 *   CHRONOS_STATUS_BANK_STREAM 0x10   streaming bank pass (CUDA-core conversion)     CHRONOS_STATUS_BANK_GEMM 0x20  fp16 grouped GEMM
 *   CHRONOS_STATUS_FP4_PROBE   0x40   chronos_b200_fp4_mma_probe                     CHRONOS_STATUS_BANK_FP4  0x80  FP4 bank passes
 *   CHRONOS_STATUS_ROUTER      0x100  router row staging                             CHRONOS_STATUS_WAIT_PROBE 0x200 chronos_b200_wait_probe
 *   CHRONOS_STATUS_GRID_SYNC   0x400  a fused decode kernel waiting for the other CTAs of its grid
 *   CHRONOS_STATUS_EP_BARRIER  0x800  chronos_b200_ep_barrier: a peer's word did not arrive
 * Read it after synchronising the stream.  Returns -1 on bad arguments.
 * No counterpart in the reference (its kernels have no device-side waits). */
#define CHRONOS_STATUS_BANK_STREAM 0x10
#define CHRONOS_STATUS_BANK_GEMM 0x20
#define CHRONOS_STATUS_FP4_PROBE 0x40
#define CHRONOS_STATUS_BANK_FP4 0x80
#define CHRONOS_STATUS_ROUTER 0x100
#define CHRONOS_STATUS_WAIT_PROBE 0x200
#define CHRONOS_STATUS_GRID_SYNC 0x400
#define CHRONOS_STATUS_EP_BARRIER 0x800
long chronos_b200_workspace_status_offset(const chronos_layer_t* layer, int n_tokens);

/* Exercises the give-up path of the library's bounded waits without any fault: a one-warp kernel waits, through the
 * same bounded wait the bank kernels use, on a shared-memory barrier that nothing will ever complete; after
 * poll_limit polls (1..4096, about a microsecond each) it raises CHRONOS_STATUS_WAIT_PROBE in *status (device int32,
 * clear it first) and returns.  No counterpart in the reference. */
int chronos_b200_wait_probe(int32_t* status, unsigned poll_limit, void* stream);

/* Message for the last non-zero status returned to the calling thread ("" if none). */
const char* chronos_b200_last_error(void);

/* Library/ABI version: increases whenever a signature or struct layout above changes. */
int chronos_b200_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif /* CHRONOS_B200_H */
