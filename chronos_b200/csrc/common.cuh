// Shared device helpers and the workspace plan of the folded-MoE forward (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "chronos_b200.h"

namespace chronos {

constexpr int kPairsPerItem = 8;  // (token, expert) pairs that share one pass over a slot's bank (= MMA N)
constexpr int kPairsPerGemmItem = 128;  // pairs of ONE expert per tensor-core work item, fp16 regime (= MMA M)
constexpr int kHealSplit = 4;           // slices of the contraction the tensor-core healer-input kernel is split into (one CTA each)
constexpr int kGroupPairs = 8;          // pairs whose bank-pass outputs one CTA of the large-batch output kernel stages in shared memory
constexpr int kDtypeF16Scaled = 2;      // internal activation source: fp16 rows already divided by the token / pair scale
constexpr int kPairsPerWideItem = 64;   // the same in the FP4 tensor regime: 3 residual terms x 64 pairs = MMA N of 192
constexpr int kWideRows = 3 * kPairsPerWideItem;           // rows of a wide activation stage image
constexpr int kWideStageBytes = kWideRows * 128 + 4 * 1024;  // 24576 B of nibbles + 4 MMAs x 2 scale blocks = 28672
constexpr int kMaxTopK = 32;
constexpr int kMaxRank = 128;
constexpr int kStageEvents = 8;   // stage boundaries of one forward call that can carry a profiling event

// Device-side view of the caller's workspace for one forward call. All offsets are 256-byte aligned.
struct Plan {
    float* logits;         // [T, E]
    int32_t* ids;          // [T, top_k]
    float* gates;          // [T, top_k]
    int32_t* offsets;      // [E + 2]  first sorted pair of expert e; entry E = shared expert; entry E+1 = total
    int32_t* cursor;       // [E + 2]  pairs of expert e already placed by the multi-CTA scatter of a large batch
    int32_t* pair_token;   // [P]      token of sorted pair p
    int32_t* pair_expert;  // [P]      expert of sorted pair p (E = shared expert)
    int32_t* pos_of;       // [T * top_k] sorted position of routing entry (t, j); -1 when skipped
    int32_t* item_start;   // [max_items] first sorted pair of work item
    int32_t* item_cnt;     // [max_items] 1..8 pairs
    int32_t* item_slot;    // [max_items] slot whose bank the item streams (n_slots = shared expert)
    int32_t* gitem_start;  // [max_gitems] tensor-core work items: up to 128 sorted pairs of one expert
    int32_t* gitem_cnt;
    int32_t* gitem_slot;
    int32_t* counters;     // [0] = number of items, [1] = number of pairs, [2] = device status word, [3] = number of gemm items,
                           // [8] = arrivals at the grid-wide hand-off of the fused decode front kernel (16 words, cleared per call)
    __half* xc;            // [P, H]   transformed gate_up inputs
    float* hmid;           // [P, r]   V_gu . x
    float* z1;             // [P, 2I]  H_r(r_s2 * (S_gu . x_c)) * scale_2
    __half* ac;            // [P, I]   transformed down inputs
    float* hpart;          // [P, I/128, r] partial V_down . act per 128-block
    float* y1;             // [P, H]   H_r(r_s2 * (S_down . a_c)) * scale_2
    float* act;            // [P, I]   SwiGLU outputs, natural order
    float* act_ss;         // [P, I/128] partial sums of squares of act
    float* tok_scale;      // [T]      power-of-two scale near rms(x[t]) (FP4 streaming regime)
    float* pscale_gu;      // [P]      scale the pair's gate_up activation image was divided by
    float* pscale_dn;      // [P]      same for the down image
    uint8_t* bq_gu;        // [max_items, H/256, 6144] FP4 activation images of the gate_up pass (NULL: not laid out)
    uint8_t* bq_dn;        // [max_items, I/256, 6144]
    float* yt;             // [P, H]   per-pair down outputs in natural row order (tensor regime only, else NULL)
    __half* x16;           // [T, H]   x / token scale as fp16 (large batches only, else NULL)
    float* tail_gu;        // [P, 2I]  tail-lattice term of the gate_up product, natural row order (NULL: layer has no tail)
    float* tail_dn;        // [P, H]   the same for the down product
    float* hsplit;         // [2 stages][kHealSplit][P, r] healer input factors, one partial sum per slice of the contraction
    __half* himg;          // [gitems][r/8][64][8] the same factors of a work item as a K-major fp16 operand tile (fused healer)
    float* heal_gu;        // [P, 2I]  healer term U_gu (V_gu x) in natural row order (fused decode path only, else NULL)
    float* heal_dn;        // [P, H]   healer term U_down (V_down act) in natural row order (fused decode path only)
    int32_t* pair_item;    // [P]      streaming work item of sorted pair p (fused decode path only)
    int32_t* pair_pos;     // [P]      position 0..7 of sorted pair p inside its work item
    float* sh8_z;          // [T, 2I]  block-FP8 shared expert: gate_up outputs (NULL: the layer has no such expert)
    __half* sh8_act;       // [T, I]   its SwiGLU outputs
    float* sh8_y;          // [T, H]   its down outputs
    int fp4_stream;        // bq_* are laid out for the FP4 streaming regime ([max_items, K/256, 6144])
    int fp4_wide;          // bq_* are laid out for the FP4 tensor regime ([max_gitems, K/256, 28672])
    int gitem_pairs;       // pairs per tensor-core work item in this call (128 or 64)
    int shared_lo, shared_n;  // tokens shared_lo .. shared_lo + shared_n - 1 also go through the shared expert
    int max_pairs;
    int max_items;
    int max_gitems;
};

struct PlanLayout {
    size_t off_logits, off_ids, off_gates, off_offsets, off_pair_token, off_pair_expert, off_pos_of, off_item_start,
        off_item_cnt, off_item_slot, off_gitem_start, off_gitem_cnt, off_gitem_slot, off_counters, off_xc, off_hmid, off_z1, off_ac, off_hpart, off_y1, off_act, off_act_ss, off_tok_scale, off_pscale_gu,
        off_pscale_dn, off_bq_gu, off_bq_dn, off_yt, off_x16, off_hsplit, off_tail_gu, off_tail_dn, off_x16t, off_heal_gu,
        off_heal_dn, off_pair_item, off_pair_pos, off_sh8_z, off_sh8_act, off_sh8_y, off_himg, total;
    int fp4, tiled, wide, tail, sh8;
    int max_pairs, max_items, max_gitems, n_bins_padded;
};

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// The always-on expert comes in one of two formats: plain NVFP4 (handled as an extra slot by the bank passes) or the
// stock block-FP8 format (csrc/shared_fp8.cu, a pass of its own).
inline bool shared_is_fp8(const chronos_layer_t& L) { return L.shared_inter > 0 && L.sh8_gu_w != nullptr; }
inline bool shared_is_nvfp4(const chronos_layer_t& L) { return L.shared_inter > 0 && L.sh8_gu_w == nullptr; }

inline PlanLayout plan_layout(const chronos_layer_t& L, int n_tokens) {
    PlanLayout p{};
    const size_t T = (size_t)n_tokens, E = (size_t)L.n_experts, k = (size_t)L.top_k, H = (size_t)L.hidden,
                 I = (size_t)L.inter, r = (size_t)L.rank;
    const size_t P = T * k + (shared_is_nvfp4(L) ? T : 0);
    p.max_pairs = (int)P;
    p.n_bins_padded = (int)(E + 2);
    p.max_items = (int)((size_t)L.n_slots + 1 + P / kPairsPerItem + 1);
    // FP4 activation images exist only for batch shapes the streaming regime serves and layers that carry re-tiled banks
    p.fp4 = (L.gu_t != nullptr && L.dn_t != nullptr && H % 256 == 0 && I % 256 == 0 && H <= 7168 && I <= 7168 &&
             T * k < 16 * (size_t)L.n_slots &&
             (!shared_is_nvfp4(L) || (L.sh_gu_t != nullptr && L.sh_dn_t != nullptr))) ? 1 : 0;
    // per-expert work items: 64 pairs in the FP4 tensor regime (128 in the fp16 one); the fused decode path cuts the
    // same lists into chunks of 8 pairs for its healer products
    p.max_gitems = (int)(E + 1 + P / (p.fp4 ? 8 : kPairsPerWideItem) + 1);
    size_t o = 0;
    auto take = [&](size_t bytes) { size_t at = o; o = align_up(o + bytes, 256); return at; };
    p.off_logits = take(T * E * 4);
    p.off_ids = take(T * k * 4);
    p.off_gates = take(T * k * 4);
    p.off_offsets = take(2 * (E + 2) * 4);  // prefix sums, then the scatter cursors of the multi-CTA plan
    p.off_pair_token = take(P * 4);
    p.off_pair_expert = take(P * 4);
    p.off_pos_of = take(T * k * 4);
    p.off_item_start = take((size_t)p.max_items * 4);
    p.off_item_cnt = take((size_t)p.max_items * 4);
    p.off_item_slot = take((size_t)p.max_items * 4);
    p.off_gitem_start = take((size_t)p.max_gitems * 4);
    p.off_gitem_cnt = take((size_t)p.max_gitems * 4);
    p.off_gitem_slot = take((size_t)p.max_gitems * 4);
    p.off_counters = take(64);
    p.off_xc = take(P * H * 2);
    p.off_hmid = take(P * r * 4);
    p.off_z1 = take(P * 2 * I * 4);
    p.off_ac = take(P * I * 2);
    p.off_hpart = take(P * (I / 128) * r * 4);
    p.off_y1 = take(P * H * 4);
    p.off_act = take(P * I * 4);
    p.off_act_ss = take(P * (I / 128) * 4);
    p.off_tok_scale = take(T * 4);
    p.off_pscale_gu = take(P * 4);
    p.off_pscale_dn = take(P * 4);
    p.tiled = (T * k >= 16 * (size_t)L.n_slots) ? 1 : 0;  // batch shapes the tensor regime serves
    // the FP4 tensor regime: re-tiled banks, the tensor-core healer path (needs healer.v_down as on disk) and its
    // shared-memory budget (4 staged vectors of 3 I or H floats)
    const bool images = L.gu_t != nullptr && L.dn_t != nullptr && H % 256 == 0 && I % 256 == 0 &&
                        (!shared_is_nvfp4(L) || (L.sh_gu_t != nullptr && L.sh_dn_t != nullptr));
    p.wide = (p.tiled && images && L.v_dn != nullptr && kGroupPairs * 3 * I * 4 <= 220 * 1024 && kGroupPairs * H * 4 <= 220 * 1024) ? 1 : 0;
    p.off_bq_gu = take(p.fp4 ? (size_t)p.max_items * (H / 256) * 6144 : (p.wide ? (size_t)p.max_gitems * (H / 256) * kWideStageBytes : 0));
    p.off_bq_dn = take(p.fp4 ? (size_t)p.max_items * (I / 256) * 6144 : (p.wide ? (size_t)p.max_gitems * (I / 256) * kWideStageBytes : 0));
    p.off_yt = take(p.tiled ? P * H * 4 : 0);
    p.off_x16 = take(p.tiled ? T * H * 2 : 0);
    p.off_hsplit = take(p.tiled ? 2 * kHealSplit * P * r * 4 : 0);
    p.off_himg = take((p.wide && L.ut_gu != nullptr) ? (size_t)p.max_gitems * kPairsPerWideItem * r * 2 : 0);
    p.off_heal_gu = take(p.fp4 ? P * 2 * I * 4 : 0);
    p.off_heal_dn = take(p.fp4 ? P * H * 4 : 0);
    p.off_pair_item = take(p.fp4 ? P * 4 : 0);
    p.off_pair_pos = take(p.fp4 ? P * 4 : 0);
    p.sh8 = shared_is_fp8(L) ? 1 : 0;
    p.off_sh8_z = take(p.sh8 ? T * 2 * I * 4 : 0);
    p.off_sh8_act = take(p.sh8 ? T * I * 2 : 0);
    p.off_sh8_y = take(p.sh8 ? T * H * 4 : 0);
    p.tail = L.tail_bits != 0 ? 1 : 0;
    p.off_tail_gu = take(p.tail ? P * 2 * I * 4 : 0);
    p.off_tail_dn = take(p.tail ? P * H * 4 : 0);
    p.off_x16t = take((p.tail && !p.tiled) ? T * H * 2 : 0);  // the fp16 token image for the tail pass when no other regime lays it out
    p.total = o;
    return p;
}

inline Plan plan_bind(const PlanLayout& l, void* ws) {
    char* b = (char*)ws;
    Plan p{};
    p.logits = (float*)(b + l.off_logits);
    p.ids = (int32_t*)(b + l.off_ids);
    p.gates = (float*)(b + l.off_gates);
    p.offsets = (int32_t*)(b + l.off_offsets);
    p.cursor = p.offsets + l.n_bins_padded;
    p.pair_token = (int32_t*)(b + l.off_pair_token);
    p.pair_expert = (int32_t*)(b + l.off_pair_expert);
    p.pos_of = (int32_t*)(b + l.off_pos_of);
    p.item_start = (int32_t*)(b + l.off_item_start);
    p.item_cnt = (int32_t*)(b + l.off_item_cnt);
    p.item_slot = (int32_t*)(b + l.off_item_slot);
    p.gitem_start = (int32_t*)(b + l.off_gitem_start);
    p.gitem_cnt = (int32_t*)(b + l.off_gitem_cnt);
    p.gitem_slot = (int32_t*)(b + l.off_gitem_slot);
    p.counters = (int32_t*)(b + l.off_counters);
    p.xc = (__half*)(b + l.off_xc);
    p.hmid = (float*)(b + l.off_hmid);
    p.z1 = (float*)(b + l.off_z1);
    p.ac = (__half*)(b + l.off_ac);
    p.hpart = (float*)(b + l.off_hpart);
    p.y1 = (float*)(b + l.off_y1);
    p.act = (float*)(b + l.off_act);
    p.act_ss = (float*)(b + l.off_act_ss);
    p.tok_scale = (float*)(b + l.off_tok_scale);
    p.pscale_gu = (float*)(b + l.off_pscale_gu);
    p.pscale_dn = (float*)(b + l.off_pscale_dn);
    p.bq_gu = (l.fp4 || l.wide) ? (uint8_t*)(b + l.off_bq_gu) : nullptr;
    p.bq_dn = (l.fp4 || l.wide) ? (uint8_t*)(b + l.off_bq_dn) : nullptr;
    p.fp4_stream = l.fp4;
    p.fp4_wide = l.wide;
    p.gitem_pairs = kPairsPerGemmItem;
    p.yt = l.tiled ? (float*)(b + l.off_yt) : nullptr;
    p.x16 = l.tiled ? (__half*)(b + l.off_x16) : nullptr;
    p.hsplit = l.tiled ? (float*)(b + l.off_hsplit) : nullptr;
    p.himg = l.wide ? (__half*)(b + l.off_himg) : nullptr;
    p.heal_gu = l.fp4 ? (float*)(b + l.off_heal_gu) : nullptr;
    p.heal_dn = l.fp4 ? (float*)(b + l.off_heal_dn) : nullptr;
    p.pair_item = l.fp4 ? (int32_t*)(b + l.off_pair_item) : nullptr;
    p.pair_pos = l.fp4 ? (int32_t*)(b + l.off_pair_pos) : nullptr;
    p.sh8_z = l.sh8 ? (float*)(b + l.off_sh8_z) : nullptr;
    p.sh8_act = l.sh8 ? (__half*)(b + l.off_sh8_act) : nullptr;
    p.sh8_y = l.sh8 ? (float*)(b + l.off_sh8_y) : nullptr;
    p.tail_gu = l.tail ? (float*)(b + l.off_tail_gu) : nullptr;
    p.tail_dn = l.tail ? (float*)(b + l.off_tail_dn) : nullptr;
    if (l.tail && !l.tiled) p.x16 = (__half*)(b + l.off_x16t);
    p.max_pairs = l.max_pairs;
    p.max_items = l.max_items;
    p.max_gitems = l.max_gitems;
    return p;
}

// Top-k selection of one routing call (shared by the router kernel and the plan kernel's fused path).
struct TopkArgs {
    const float* logits;   // [T, E]; NULL = no top-k to run
    const float* e_bias;   // [E] or NULL
    int kind, renorm;
    float scaling;
    int n_tokens, n_experts, top_k;
    int32_t* ids;          // [T, top_k]
    float* gates;          // [T, top_k]
};

// ---- host-side launch wrappers (one per .cu file) -------------------------------------------------------------
int launch_dequant(const uint8_t* packed, const uint8_t* scale, const float* s2, float* out, int rows, int cols,
                   cudaStream_t st);
int launch_unfold(const chronos_layer_t& L, int expert, int which, float* out, float* scratch, cudaStream_t st);
int launch_unfold_static(const chronos_layer_t& L, int expert, int which, float* out, cudaStream_t st);
int launch_router(const chronos_layer_t& L, const void* x, int x_dtype, int n_tokens, int32_t* ids, float* gates,
                  float* logits, float* tok_scale, int32_t* status, cudaStream_t st);
int launch_coalesced_topk(const chronos_layer_t& L, const float* logits, int n_tokens, int tps, int pool, int keep, float bonus,
                          int32_t* ids, float* gates, cudaStream_t st);
int launch_plan(const chronos_layer_t& L, const int32_t* ids, int n_tokens, int with_shared, int reset_status,
                const TopkArgs& tk, const Plan& p, cudaStream_t st);
int launch_token_scale(const void* x, int x_dtype, int n_tokens, int hidden, float* tok_scale, cudaStream_t st);
int launch_tokens_f16(const void* x, int x_dtype, int n_tokens, int hidden, const float* tok_scale, __half* x16, cudaStream_t st);
int launch_pre_gu(const chronos_layer_t& L, const void* x, int x_dtype, const Plan& p, int fp4, int many_pairs,
                  cudaStream_t st);
int launch_combine_tiled(const chronos_layer_t& L, const Plan& p, const float* gates, int n_tokens, int with_shared, void* y,
                         int y_dtype, cudaStream_t st);
int launch_mid(const chronos_layer_t& L, const Plan& p, int fp4, cudaStream_t st);
// tensor-core healer path for batches with many pairs per expert (csrc/healer_mma.cu)
bool healer_mma_fits(const chronos_layer_t& L);
int launch_healer_in_mma(const chronos_layer_t& L, int stage, const void* x, int x_dtype, const Plan& p, cudaStream_t st);
int launch_mid_mma(const chronos_layer_t& L, const Plan& p, int wide, cudaStream_t st);
// tail lattice (csrc/tail.cu)
int launch_tail_pass(const chronos_layer_t& L, int stage, const void* x, int x_dtype, const Plan& p, cudaStream_t st);
int launch_tail_add(const chronos_layer_t& L, int expert, int which, float* out, cudaStream_t st);
int launch_bank_fp4_wide(const chronos_layer_t& L, int stage /*0 gu, 1 down*/, const Plan& p, cudaStream_t st);
int launch_down_out_mma(const chronos_layer_t& L, const Plan& p, cudaStream_t st);
int launch_heal_image(const chronos_layer_t& L, int stage, const Plan& p, cudaStream_t st);
bool healer_fused(const chronos_layer_t& L, const Plan& p);
int launch_mid_fused(const chronos_layer_t& L, const Plan& p, cudaStream_t st);
bool combine_gather_fits(const chronos_layer_t& L);
int launch_combine_gather(const chronos_layer_t& L, const Plan& p, const float* gates, int n_tokens, int with_shared, void* y,
                          int y_dtype, cudaStream_t st);
int launch_combine_sum(const chronos_layer_t& L, const Plan& p, const float* gates, int n_tokens, int with_shared, void* y,
                       int y_dtype, cudaStream_t st);
int launch_combine(const chronos_layer_t& L, const Plan& p, const float* gates, int n_tokens, int with_shared, void* y,
                   int y_dtype, cudaStream_t st);
int launch_bank_stream(const chronos_layer_t& L, int stage /*0 gu, 1 down*/, const Plan& p, cudaStream_t st);
int launch_bank_fp4(const chronos_layer_t& L, int stage /*0 gu, 1 down*/, const Plan& p, cudaStream_t st);
int launch_bank_gemm(const chronos_layer_t& L, int stage /*0 gu, 1 down*/, const Plan& p, cudaStream_t st);
// fused decode path (csrc/decode_fused.cu): front kernel (router, top-k, coalescing, gate_up input), the kernels between and
// after the bank passes; the healer products ride along inside the bank passes (side warps of bank_fp4_kernel)
bool decode_fused_fits(const chronos_layer_t& L, int x_dtype, int n_tokens, const Plan& p);
int launch_decode_front(const chronos_layer_t& L, const void* x, int x_dtype, int n_tokens, const int32_t* ids_in,
                        int with_shared, const Plan& p, cudaStream_t st);
int launch_decode_mid(const chronos_layer_t& L, const Plan& p, cudaStream_t st);
int launch_decode_combine(const chronos_layer_t& L, const Plan& p, const int32_t* ids, const float* gates, int n_tokens, int with_shared,
                          void* y, int y_dtype, cudaStream_t st);
int launch_bank_fp4_fused(const chronos_layer_t& L, int stage /*0 gu, 1 down*/, const Plan& p, const void* x, int x_dtype, cudaStream_t st);
// expert-parallel dispatch / combine helpers (csrc/ep_kernels.cu)
int launch_ep_pack(const void* x, int x_dtype, const int32_t* ids, const float* gates, int n_tokens, int top_k, int hidden,
                   int world, int experts_per_rank, int capacity, void* send_rows, int32_t* send_meta, int32_t* slot_of,
                   int32_t* overflow, int block_rows, long meta_block_ints, cudaStream_t st);
int launch_ep_unpack_meta(const int32_t* meta, int world, int capacity, int top_k, int32_t* ids_out, float* gates_out, int block_rows,
                          long meta_block_ints, int tail_rows, cudaStream_t st);
int launch_ep_combine(const void* back, int dtype, const int32_t* slot_of, const void* extra, int n_tokens, int hidden, int world,
                      int capacity, void* y, int y_dtype, int block_rows, cudaStream_t st);
int launch_ep_pack_peer(const void* x, int x_dtype, const int32_t* ids, const float* gates, int n_tokens, int top_k, int hidden,
                        int world, int experts_per_rank, int capacity, void* const* peer_bases, int my_rank, int block_rows,
                        int32_t* slot_of, int32_t* overflow, cudaStream_t st);
int launch_ep_send_back_peer(const void* part, int dtype, int hidden, int world, int block_rows, int capacity, int top_k, const void* recv_base,
                             void* const* peer_back, int my_rank, cudaStream_t st);
int launch_ep_barrier(void* const* pads, int my_rank, int world, uint32_t epoch, int32_t* status, cudaStream_t st);
int launch_dequant_fp8_block(const uint8_t* w, const float* s, float* out, int rows, int cols, cudaStream_t st);
int launch_shared_fp8(const chronos_layer_t& L, const void* x, int x_dtype, const Plan& p, int first, int count, void* y, int y_dtype,
                      cudaStream_t st);
int launch_wait_probe(int32_t* status, uint32_t poll_limit, cudaStream_t st);
int launch_fp4_probe(const uint8_t* a_img, const uint8_t* b_img, int n_stages, int b_rows, float* d_out, int32_t* status,
                     cudaStream_t st);
int launch_residual_rmsnorm(void* h, const void* y, const float* w, void* xn, int dtype, int n_tokens, int hidden,
                            float eps, cudaStream_t st);

void set_error(const char* fmt, ...);
int check_launch(const char* what);
int device_sm_count();  // SMs of the current device (cached per device)
// CTAs a streaming FP4 bank pass is launched with (stage 0: gate_up, 1: down)
inline int bank_fp4_grid(const chronos_layer_t& L, int stage, const Plan& p) {
    const long max_tiles = (long)p.max_items * ((stage == 0 ? 2 * L.inter : L.hidden) / 128);
    const int sms = device_sm_count();
    return (int)(max_tiles < sms ? max_tiles : sms);
}
int ensure_dynamic_smem(const void* func, size_t bytes, const char* what);  // shared-memory opt-in, cached per (kernel, device)

#ifdef __CUDACC__
// ---- device helpers ---------------------------------------------------------------------------------------------

__device__ __forceinline__ float ld_act(const void* x, int dtype, size_t i) {
    if (dtype == kDtypeF16Scaled) return __half2float(((const __half*)x)[i]);
    return dtype == CHRONOS_DTYPE_BF16 ? __bfloat162float(((const __nv_bfloat16*)x)[i]) : ((const float*)x)[i];
}

// 16 consecutive activations starting at element i (i a multiple of 16) as fp32.
__device__ __forceinline__ void ld_act16(const void* x, int dtype, size_t i, float (&out)[16]) {
    if (dtype == CHRONOS_DTYPE_BF16) {
        const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(x) + i);
        const uint4 a = src[0], b = src[1];
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            out[2 * q] = __uint_as_float(w[q] << 16);
            out[2 * q + 1] = __uint_as_float(w[q] & 0xffff0000u);
        }
    } else {
        const float4* src = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + i);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 v = src[q];
            out[4 * q] = v.x; out[4 * q + 1] = v.y; out[4 * q + 2] = v.z; out[4 * q + 3] = v.w;
        }
    }
}

// Two e4m3 bytes (low byte first) -> two fp32 values. Exact: every e4m3 value is representable in fp16.
__device__ __forceinline__ float2 e4m3x2_to_f32(uint16_t v) {
    uint32_t h2;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(v));
    return __half22float2(*reinterpret_cast<__half2*>(&h2));
}
__device__ __forceinline__ float e4m3_to_f32(uint8_t v) { return e4m3x2_to_f32((uint16_t)v).x; }

// Four bytes = eight e2m1 nibbles -> four f16x2 registers; low nibble of each byte lands in the low half.
__device__ __forceinline__ void e2m1x8_to_f16x2(uint32_t w, uint32_t& h0, uint32_t& h1, uint32_t& h2, uint32_t& h3) {
    asm("{\n"
        ".reg .b8 b0, b1, b2, b3;\n"
        "mov.b32 {b0, b1, b2, b3}, %4;\n"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n"
        "cvt.rn.f16x2.e2m1x2 %1, b1;\n"
        "cvt.rn.f16x2.e2m1x2 %2, b2;\n"
        "cvt.rn.f16x2.e2m1x2 %3, b3;\n"
        "}\n"
        : "=r"(h0), "=r"(h1), "=r"(h2), "=r"(h3)
        : "r"(w));
}

// Orthonormal 128-point Walsh-Hadamard transform (Sylvester order, scale 1/sqrt(128)) of a vector spread over a
// warp: lane l holds elements 4l .. 4l+3. Same matrix as build_hadamard_128
// (chronos_1t/converter/convert_glm53_flash_colab.py:41-45).
__device__ __forceinline__ void fwht128_warp(float (&v)[4], int lane) {
    float a = v[0] + v[1], b = v[0] - v[1], c = v[2] + v[3], d = v[2] - v[3];
    v[0] = a + c; v[1] = b + d; v[2] = a - c; v[3] = b - d;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        const float sg = (lane & m) ? -1.0f : 1.0f;  // partner - own in the upper half, own + partner in the lower: one FMA
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float o = __shfl_xor_sync(0xffffffffu, v[i], m);
            v[i] = __fmaf_rn(v[i], sg, o);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] *= 0.08838834764831845f;
}

// The same transform with a 128-block per HALF-warp: lane jl = lane & 15 holds elements 8 jl .. 8 jl + 7 of the block of
// its half-warp (a warp then covers a 256-column stage). The butterfly stages run in the same order (element bits 0 .. 6)
// with the same operands, so the results are bit-identical to fwht128_warp; three stages are in-lane and four cross
// lanes, and everything per lane (scales, addresses, stores) is amortised over eight values instead of four.
__device__ __forceinline__ void fwht128_half(float (&v)[8], int lane) {
#pragma unroll
    for (int s = 1; s < 8; s <<= 1)
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (!(i & s)) {
                const float a = v[i], b = v[i | s];
                v[i] = a + b;
                v[i | s] = a - b;
            }
#pragma unroll
    for (int m = 1; m < 16; m <<= 1) {
        const float sg = (lane & m) ? -1.0f : 1.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float o = __shfl_xor_sync(0xffffffffu, v[i], m);
            v[i] = __fmaf_rn(v[i], sg, o);
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] *= 0.08838834764831845f;
}

// softplus as torch evaluates it (F.softplus, beta 1, threshold 20): x above the threshold passes through.
__device__ __forceinline__ float softplus_f32(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

// Router flavours. choice = the score the top-k ranks by; weight source = the unbiased score the gate is made from.
//   softmax top-k     (chronos_1t/models/vllm_chronos_moe.py:310-314): both are the logit; gate = softmax over the k chosen
//   sigmoid noaux_tc  (chronos_1t/models/glm53_chronos_moe.py:392-399): sigmoid(logit) (+ bias for the choice)
//   sqrt-softplus     (chronos_1t/models/dsv41_chronos_moe.py:3402-3410): sqrt(softplus(logit)) (+ bias for the choice)
__device__ __forceinline__ float router_weight_source(const TopkArgs& a, float lg) {
    if (a.kind == CHRONOS_ROUTER_SIGMOID_NOAUX) return 1.0f / (1.0f + expf(-lg));
    if (a.kind == CHRONOS_ROUTER_SQRT_SOFTPLUS) return sqrtf(softplus_f32(lg));
    return lg;
}
__device__ __forceinline__ float router_choice(const TopkArgs& a, float lg, int e) {
    const float s = router_weight_source(a, lg);
    return a.kind == CHRONOS_ROUTER_SOFTMAX_TOPK ? s : s + (a.e_bias ? a.e_bias[e] : 0.0f);
}

// k rounds of warp arg-max for token t (ties -> lower index) and the gate weights; executed by one full warp.
// A candidate whose choice score is NaN (a NaN activation row makes every logit NaN) or -inf (a -inf bias entry) can
// never win a round. When no candidate is left the round emits id -1 with gate 0 - an entry every consumer skips -
// so no index outside [0, n_experts) is ever formed or used as an address.
constexpr int kNoExpert = 0x7fffffff;

// Largest of a lane's PL candidates (candidate i = expert i * 32 + lane; absent or spent ones hold -inf) and its expert id,
// ties to the lower id, kNoExpert when all are -inf. A pairwise tree: the dependent chain is log2(PL) selects long.
template <int PL>
__device__ __forceinline__ void lane_argmax(const float (&choice)[PL], int lane, float& best, int& best_e) {
    float v[PL];
    int id[PL];
#pragma unroll
    for (int i = 0; i < PL; ++i) { v[i] = choice[i]; id[i] = i; }
#pragma unroll
    for (int stride = 1; stride < PL; stride *= 2)
#pragma unroll
        for (int i = 0; i + stride < PL; i += 2 * stride)
            if (v[i + stride] > v[i]) { v[i] = v[i + stride]; id[i] = id[i + stride]; }  // equal: the lower index stays
    best = v[0];
    best_e = v[0] > -INFINITY ? id[0] * 32 + lane : kNoExpert;
}

template <int PL>
__device__ __forceinline__ void topk_one_token_pl(const TopkArgs& a, int t, int lane) {
    float choice[PL];
#pragma unroll
    for (int i = 0; i < PL; ++i) {
        const int e = i * 32 + lane;
        float c = -INFINITY;
        if (e < a.n_experts) {
            const float lg = a.logits[(size_t)t * a.n_experts + e];
            c = router_choice(a, lg, e);
            if (!(c == c)) c = -INFINITY;  // NaN never wins
        }
        choice[i] = c;
    }
    float my_val = 0.0f;  // lane j keeps the j-th chosen weight source
    int my_id = -1;
    for (int j = 0; j < a.top_k; ++j) {
        float best;
        int best_e;
        lane_argmax<PL>(choice, lane, best, best_e);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, off);
            const int oe = __shfl_xor_sync(0xffffffffu, best_e, off);
            if (ov > best || (ov == best && oe < best_e)) { best = ov; best_e = oe; }
        }
        const bool found = best_e != kNoExpert;  // warp-uniform
#pragma unroll
        for (int i = 0; i < PL; ++i)
            if (found && i * 32 + lane == best_e) choice[i] = -INFINITY;  // remove the winner from its owner lane
        if (lane == j && found) my_id = best_e;
    }
    // lane j fetches the logit of its winner once, after the rounds: a load inside the loop would make every round wait
    // for the previous round's load (they would all target the same register)
    const bool have = lane < a.top_k && my_id >= 0;
    if (have) my_val = router_weight_source(a, a.logits[(size_t)t * a.n_experts + my_id]);
    float gate;
    if (a.kind != CHRONOS_ROUTER_SOFTMAX_TOPK) {
        const float s = have ? my_val : 0.0f;
        float tot = 0.0f;  // sequential sum in index order, the way a row reduction over k values reads
        for (int j = 0; j < a.top_k; ++j) tot += __shfl_sync(0xffffffffu, s, j);
        gate = a.renorm ? my_val / (tot + 1e-20f) : my_val;
        gate *= a.scaling;
    } else {
        const float mx = __shfl_sync(0xffffffffu, my_val, 0);  // chosen values are in descending order
        const float ex = have ? expf(my_val - mx) : 0.0f;
        float tot = 0.0f;
        for (int j = 0; j < a.top_k; ++j) tot += __shfl_sync(0xffffffffu, ex, j);
        gate = ex / tot;
    }
    if (lane < a.top_k) {
        a.ids[(size_t)t * a.top_k + lane] = my_id;
        a.gates[(size_t)t * a.top_k + lane] = have ? gate : 0.0f;
    }
}
__device__ __forceinline__ void topk_one_token(const TopkArgs& a, int t, int lane) {
    if (a.n_experts <= 256) topk_one_token_pl<8>(a, t, lane);
    else if (a.n_experts <= 320) topk_one_token_pl<10>(a, t, lane);
    else if (a.n_experts <= 512) topk_one_token_pl<16>(a, t, lane);
    else topk_one_token_pl<32>(a, t, lane);
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// z * sigmoid(z) with the fast exponential and division (relative error ~1e-6, far inside the layer tolerance)
__device__ __forceinline__ float silu_f32(float z) { return __fdividef(z, 1.0f + __expf(-z)); }

__device__ __forceinline__ __half f32_to_f16_sat(float v) {
    unsigned short r;
    asm("cvt.rn.satfinite.f16.f32 %0, %1;" : "=h"(r) : "f"(v));
    return __ushort_as_half(r);
}
// ---- warp-level tensor-core helpers of the healer products (mma.sync m16n8k16, fp16 operands, fp32 accumulate) ------
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t v16) {
    uint32_t r;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"((uint16_t)v16));
    return r;
}
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_f16x2_sat(float lo, float hi) {
    const __half2 h = __halves2half2(f32_to_f16_sat(lo), f32_to_f16_sat(hi));
    return *reinterpret_cast<const uint32_t*>(&h);
}

// ---------------------------------------------------------------------------------------------------------------
// FP4 quantiser: a 128-block of activations (lane l holds elements 4l..4l+3, already divided by the pair's scale) is
// written as three residual e2m1 terms with ue4m3 scales per 16 elements into an activation stage image
// (csrc/bank_fp4.cu describes the image): term t quantises the residual times 32^t, so the tensor-core column of
// term t is worth 32^-t. Row of the image = t * TSTRIDE + p (p = the pair's position in its work item).
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t f32x2_to_e4m3x2(float lo, float hi) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %2, %1;" : "=h"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ uint32_t f32x2_to_e2m1x2(float lo, float hi) {
    uint16_t r;
    asm("{\n.reg .b8 t;\ncvt.rn.satfinite.e2m1x2.f32 t, %2, %1;\nmov.b16 %0, {t, 0};\n}" : "=h"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float2 e2m1x2_to_f32(uint32_t byte) {
    uint32_t h2;
    asm("{\n.reg .b8 t, z;\nmov.b16 {t, z}, %1;\ncvt.rn.f16x2.e2m1x2 %0, t;\n}" : "=r"(h2) : "h"((uint16_t)byte));
    return __half22float2(*reinterpret_cast<__half2*>(&h2));
}

template <int ROWS, int TSTRIDE>  // rows of the stage image (32 streaming, 192 tensor regime); row of term t = t * TSTRIDE + prow
__device__ __forceinline__ void quantize_block_fp4x3(const float (&v)[4], int lane, uint8_t* __restrict__ stage_img,
                                                     int half, int prow) {
    constexpr int SFJ = 512 * ((ROWS + 127) / 128);  // scale bytes of one MMA (64 columns): a 512-byte block per 128 rows
    float r[4] = {v[0], v[1], v[2], v[3]};
    const int c = half * 4 + (lane >> 3), b = 2 * (lane & 7);
    const int j = half * 2 + (lane >> 4), sidx = (lane & 15) >> 2;
#pragma unroll
    for (int t = 0; t < 3; ++t) {
        const float up = t == 0 ? 1.0f : (t == 1 ? 32.0f : 1024.0f);
        float m = fmaxf(fmaxf(fabsf(r[0]), fabsf(r[1])), fmaxf(fabsf(r[2]), fabsf(r[3])));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
        const uint32_t sc8 = f32x2_to_e4m3x2(m * up * (1.0f / 6.0f), 0.0f) & 0xffu;
        const float sdec = e4m3_to_f32((uint8_t)sc8);
        // approximate reciprocal: inv only positions the values for rounding; the residual is taken from what was stored
        const float inv = sdec > 0.0f ? __fdividef(up, sdec) : 0.0f;
        const uint32_t b01 = f32x2_to_e2m1x2(r[0] * inv, r[1] * inv) & 0xffu;
        const uint32_t b23 = f32x2_to_e2m1x2(r[2] * inv, r[3] * inv) & 0xffu;
        const float2 q01 = e2m1x2_to_f32(b01), q23 = e2m1x2_to_f32(b23);
        const float back = sdec * (1.0f / up);  // exact: up is a power of two
        r[0] = fmaf(-q01.x, back, r[0]); r[1] = fmaf(-q01.y, back, r[1]);
        r[2] = fmaf(-q23.x, back, r[2]); r[3] = fmaf(-q23.y, back, r[3]);
        const int n = t * TSTRIDE + prow;
        *reinterpret_cast<uint16_t*>(stage_img + c * (ROWS * 16) + n * 16 + b) = (uint16_t)(b01 | (b23 << 8));
        if ((lane & 3) == 0)
            stage_img[ROWS * 128 + j * SFJ + (n >> 7) * 512 + (n & 31) * 16 + ((n & 127) >> 5) * 4 + sidx] = (uint8_t)sc8;
    }
}

// The same quantiser for a whole 256-column stage per warp: lane (half = lane >> 4, jl = lane & 15) holds elements
// 8 jl .. 8 jl + 7 of 128-block `half` of the stage (the layout fwht128_half leaves). Same arithmetic per 16-element scale
// block (two lanes instead of four), same bytes; 4-byte nibble stores.
template <int ROWS, int TSTRIDE>
__device__ __forceinline__ void quantize_stage_fp4x3(const float (&v)[8], int lane, uint8_t* __restrict__ stage_img, int prow) {
    constexpr int SFJ = 512 * ((ROWS + 127) / 128);
    float r[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) r[i] = v[i];
    const int half = lane >> 4, jl = lane & 15;
    const int c = half * 4 + (jl >> 2), b = 4 * (jl & 3);
    const int j = half * 2 + (jl >> 3), sidx = (jl & 7) >> 1;
#pragma unroll
    for (int t = 0; t < 3; ++t) {
        const float up = t == 0 ? 1.0f : (t == 1 ? 32.0f : 1024.0f);
        float m = fmaxf(fmaxf(fmaxf(fabsf(r[0]), fabsf(r[1])), fmaxf(fabsf(r[2]), fabsf(r[3]))),
                        fmaxf(fmaxf(fabsf(r[4]), fabsf(r[5])), fmaxf(fabsf(r[6]), fabsf(r[7]))));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        const uint32_t sc8 = f32x2_to_e4m3x2(m * up * (1.0f / 6.0f), 0.0f) & 0xffu;
        const float sdec = e4m3_to_f32((uint8_t)sc8);
        const float inv = sdec > 0.0f ? __fdividef(up, sdec) : 0.0f;
        const float back = sdec * (1.0f / up);  // exact: up is a power of two
        uint32_t word = 0u;
#pragma unroll
        for (int h2 = 0; h2 < 4; ++h2) {
            const uint32_t byte = f32x2_to_e2m1x2(r[2 * h2] * inv, r[2 * h2 + 1] * inv) & 0xffu;
            const float2 q = e2m1x2_to_f32(byte);
            r[2 * h2] = fmaf(-q.x, back, r[2 * h2]);
            r[2 * h2 + 1] = fmaf(-q.y, back, r[2 * h2 + 1]);
            word |= byte << (8 * h2);
        }
        const int n = t * TSTRIDE + prow;
        *reinterpret_cast<uint32_t*>(stage_img + c * (ROWS * 16) + n * 16 + b) = word;
        if ((jl & 1) == 0)
            stage_img[ROWS * 128 + j * SFJ + (n >> 7) * 512 + (n & 31) * 16 + ((n & 127) >> 5) * 4 + sidx] = (uint8_t)sc8;
    }
}

// Power-of-two scale near the root mean square of a vector (1 when the vector is all zero).
__device__ __forceinline__ float pow2_scale(float sumsq, int n) {
    const float rms = sqrtf(sumsq / (float)n);
    return rms > 0.0f ? exp2f(rintf(log2f(rms))) : 1.0f;
}

// One 128-block of a gate_up input: gather + sign, Walsh-Hadamard, sign (identity for the shared expert).
__device__ __forceinline__ void transform_gu_block(const chronos_layer_t& L, const void* __restrict__ x, int x_dtype,
                                                   int t, int e, int blk, int lane, float (&v)[4]) {
    const int H = L.hidden;
    if (e >= L.n_experts) {  // shared expert: plain weights, identity keys
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = ld_act(x, x_dtype, (size_t)t * H + blk * 128 + lane * 4 + i);
        return;
    }
    const uint2 ce = *reinterpret_cast<const uint2*>(L.gu_cin + (size_t)e * H + blk * 128 + lane * 4);
    const uint32_t ent[4] = {ce.x & 0xffffu, ce.x >> 16, ce.y & 0xffffu, ce.y >> 16};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float xv = ld_act(x, x_dtype, (size_t)t * H + (ent[i] & 0x7fffu));
        v[i] = (ent[i] >> 15) ? -xv : xv;
    }
    fwht128_warp(v, lane);
    const uint32_t sw = L.gu_cs2[(size_t)e * (H / 32) + blk * 4 + lane / 8] >> ((lane & 7) * 4);
#pragma unroll
    for (int i = 0; i < 4; ++i)
        if ((sw >> i) & 1u) v[i] = -v[i];
}

// One 128-block of a down input from the SwiGLU outputs `act` (fp32, natural order) of the pair.
__device__ __forceinline__ void transform_dn_block(const chronos_layer_t& L, const float* __restrict__ act, int e, int blk,
                                                   int lane, float (&v)[4]) {
    const int I = L.inter;
    if (e >= L.n_experts) {
        const float4 a = *reinterpret_cast<const float4*>(act + blk * 128 + lane * 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        return;
    }
    const uint2 ce = *reinterpret_cast<const uint2*>(L.dn_cin + (size_t)e * I + blk * 128 + lane * 4);
    const uint32_t ent[4] = {ce.x & 0xffffu, ce.x >> 16, ce.y & 0xffffu, ce.y >> 16};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float a = act[ent[i] & 0x7fffu];
        v[i] = (ent[i] >> 15) ? -a : a;
    }
    fwht128_warp(v, lane);
    const uint32_t sw = L.dn_cs2[(size_t)e * (I / 32) + blk * 4 + lane / 8] >> ((lane & 7) * 4);
#pragma unroll
    for (int i = 0; i < 4; ++i)
        if ((sw >> i) & 1u) v[i] = -v[i];
}

// A whole 256-column stage per warp (half-warp = 128-block, lane jl holds elements 8 jl .. 8 jl + 7): the same values as
// two calls of the block forms above, with the per-lane work amortised over eight elements.
__device__ __forceinline__ void transform_gu_stage(const chronos_layer_t& L, const void* __restrict__ x, int x_dtype, int t, int e,
                                                   int st, int lane, float (&v)[8]) {
    const int H = L.hidden, half = lane >> 4, jl = lane & 15;
    const int k0 = st * 256 + half * 128 + jl * 8;
    if (e >= L.n_experts) {  // shared expert: plain weights, identity keys
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = ld_act(x, x_dtype, (size_t)t * H + k0 + i);
        return;
    }
    const uint4 ce = *reinterpret_cast<const uint4*>(L.gu_cin + (size_t)e * H + k0);
    const uint32_t ent[8] = {ce.x & 0xffffu, ce.x >> 16, ce.y & 0xffffu, ce.y >> 16, ce.z & 0xffffu, ce.z >> 16, ce.w & 0xffffu, ce.w >> 16};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float xv = ld_act(x, x_dtype, (size_t)t * H + (ent[i] & 0x7fffu));
        v[i] = (ent[i] >> 15) ? -xv : xv;
    }
    fwht128_half(v, lane);
    const uint32_t sw = L.gu_cs2[(size_t)e * (H / 32) + st * 8 + half * 4 + (jl >> 2)] >> ((jl & 3) * 8);
#pragma unroll
    for (int i = 0; i < 8; ++i)
        if ((sw >> i) & 1u) v[i] = -v[i];
}

__device__ __forceinline__ void transform_dn_stage(const chronos_layer_t& L, const float* __restrict__ act, int e, int st, int lane,
                                                   float (&v)[8]) {
    const int I = L.inter, half = lane >> 4, jl = lane & 15;
    const int k0 = st * 256 + half * 128 + jl * 8;
    if (e >= L.n_experts) {
        const float4 a0 = *reinterpret_cast<const float4*>(act + k0), a1 = *reinterpret_cast<const float4*>(act + k0 + 4);
        v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w; v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
        return;
    }
    const uint4 ce = *reinterpret_cast<const uint4*>(L.dn_cin + (size_t)e * I + k0);
    const uint32_t ent[8] = {ce.x & 0xffffu, ce.x >> 16, ce.y & 0xffffu, ce.y >> 16, ce.z & 0xffffu, ce.z >> 16, ce.w & 0xffffu, ce.w >> 16};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float a = act[ent[i] & 0x7fffu];
        v[i] = (ent[i] >> 15) ? -a : a;
    }
    fwht128_half(v, lane);
    const uint32_t sw = L.dn_cs2[(size_t)e * (I / 32) + st * 8 + half * 4 + (jl >> 2)] >> ((jl & 3) * 8);
#pragma unroll
    for (int i = 0; i < 8; ++i)
        if ((sw >> i) & 1u) v[i] = -v[i];
}

__device__ __forceinline__ void store_half4(__half* dst, const float (&v)[4]) {
    __half2 h01 = __halves2half2(f32_to_f16_sat(v[0]), f32_to_f16_sat(v[1]));
    __half2 h23 = __halves2half2(f32_to_f16_sat(v[2]), f32_to_f16_sat(v[3]));
    uint2 o;
    o.x = *reinterpret_cast<uint32_t*>(&h01);
    o.y = *reinterpret_cast<uint32_t*>(&h23);
    *reinterpret_cast<uint2*>(dst) = o;
}


constexpr uint32_t kWaitLimit = 1u << 20;  // polls of a ~1 us bounded try_wait before giving up: about a second

// Bits of the device status word (counters[2] of the workspace; the probes take a status pointer of their own).
constexpr int kStatusBankStreamTimeout = 0x10;   // bank_stream_kernel: a ring wait expired
constexpr int kStatusBankGemmTimeout = 0x20;     // bank_gemm_kernel
constexpr int kStatusFp4ProbeTimeout = 0x40;     // fp4_mma_probe_kernel
constexpr int kStatusEpBarrierTimeout = 0x800;     // ep_barrier_kernel: a peer's word did not arrive
constexpr int kStatusBankFp4Timeout = 0x80;      // bank_fp4_kernel / bank_fp4_wide_kernel
constexpr int kStatusRouterTimeout = 0x100;      // router_logits_small_kernel: staged rows never arrived
constexpr int kStatusWaitProbeTimeout = 0x200;   // wait_probe_kernel: the wait it is built to lose
constexpr int kStatusGridSyncTimeout = 0x400;    // a fused decode kernel gave up waiting for the other CTAs of its grid

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// Bounded wait: returns false when the phase did not complete within the poll limit.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint32_t limit = kWaitLimit) {
    for (uint32_t it = 0; it < limit; ++it) {
        uint32_t ok;
        asm volatile(
            "{\n.reg .pred p;\n"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 1000;\n"
            "selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    return false;
}
// One non-blocking test of a phase.
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n.reg .pred p;\n"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        "selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
// Streamed-once data (bank bytes) is tagged evict-first in L2 so that it does not push out the small tensors the other
// kernels of the layer re-read (router weights, key tables, activations, scratch).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void bulk_g2s_stream(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar, uint64_t pol) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar), "l"(pol)
                 : "memory");
}
#endif  // __CUDACC__

}  // namespace chronos
