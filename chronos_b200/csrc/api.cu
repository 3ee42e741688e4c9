// extern "C" entry points of libchronos_b200.so: argument validation on the host, then stream-ordered launches.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace chronos {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

int check_launch(const char* what) {
    const cudaError_t rc = cudaGetLastError();
    if (rc == cudaSuccess) return CHRONOS_OK;
    set_error("%s: %s", what, cudaGetErrorString(rc));
    return CHRONOS_E_LAUNCH;
}

// ---- per-device launch facts, looked up once -----------------------------------------------------------------
// The SM count and the dynamic shared-memory opt-in of a kernel do not change while the process lives; asking the
// runtime for them on every launch costs several driver calls per layer on the host side of a ~100 us step.
constexpr int kMaxDevices = 64;
static std::mutex g_cache_mu;
static int g_sm_count[kMaxDevices];

static int current_device() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
    return dev;
}

int device_sm_count() {
    const int dev = current_device();
    if (dev < 0) return 148;
    std::lock_guard<std::mutex> lock(g_cache_mu);
    if (g_sm_count[dev] == 0) {
        int sms = 148;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) { cudaGetLastError(); sms = 148; }
        g_sm_count[dev] = sms;
    }
    return g_sm_count[dev];
}

struct SmemOptIn { const void* func; int dev; size_t bytes; };
static SmemOptIn g_optin[256];
static int g_n_optin = 0;

// Makes sure `func` may be launched with `bytes` of dynamic shared memory on the current device; the runtime is asked
// only when a (kernel, device) pair needs more than it was granted before.
int ensure_dynamic_smem(const void* func, size_t bytes, const char* what) {
    const int dev = current_device();
    std::lock_guard<std::mutex> lock(g_cache_mu);
    SmemOptIn* slot = nullptr;
    for (int i = 0; i < g_n_optin; ++i)
        if (g_optin[i].func == func && g_optin[i].dev == dev) { slot = &g_optin[i]; break; }
    if (slot != nullptr && slot->bytes >= bytes) return CHRONOS_OK;
    const cudaError_t rc = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (rc != cudaSuccess) {
        cudaGetLastError();
        set_error("%s: cannot opt in to %zu bytes of shared memory: %s", what, bytes, cudaGetErrorString(rc));
        return CHRONOS_E_LAUNCH;
    }
    if (slot == nullptr && g_n_optin < 256 && dev >= 0) slot = &g_optin[g_n_optin++];
    if (slot != nullptr) *slot = SmemOptIn{func, dev, bytes};
    return CHRONOS_OK;
}

static bool aligned16(const void* p) { return p != nullptr && (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int validate_layer(const chronos_layer_t* L, bool need_router) {
    if (!L) { set_error("layer is NULL"); return CHRONOS_E_ALIGN; }
    if (L->hidden <= 0 || L->inter <= 0 || L->hidden % 128 || L->inter % 128 || L->hidden > 32768 || 2 * L->inter > 32768) {
        set_error("hidden (%d) and inter (%d) must be positive multiples of 128 with hidden, 2*inter <= 32768", L->hidden, L->inter);
        return CHRONOS_E_SHAPE;
    }
    if (L->group_size <= 0 || L->n_slots <= 0 || L->n_experts != L->n_slots * L->group_size || L->n_experts > 1024) {
        set_error("n_experts (%d) must equal n_slots (%d) * group_size (%d) and be <= 1024", L->n_experts, L->n_slots, L->group_size);
        return CHRONOS_E_SHAPE;
    }
    if (L->rank != 16 && L->rank != 32 && L->rank != 64 && L->rank != 128) {
        set_error("healer rank (%d) must be 16, 32, 64 or 128", L->rank);
        return CHRONOS_E_SHAPE;
    }
    if (L->top_k <= 0 || L->top_k > kMaxTopK || L->top_k > L->n_experts) {
        set_error("top_k (%d) must be in [1, min(%d, n_experts)]", L->top_k, kMaxTopK);
        return CHRONOS_E_SHAPE;
    }
    if (L->shared_inter != 0 && L->shared_inter != L->inter) {
        set_error("shared_inter (%d) must be 0 or equal to inter (%d)", L->shared_inter, L->inter);
        return CHRONOS_E_SHAPE;
    }
    if (L->router_kind < CHRONOS_ROUTER_SOFTMAX_TOPK || L->router_kind > CHRONOS_ROUTER_SQRT_SOFTPLUS) {
        set_error("router_kind %d is not a CHRONOS_ROUTER_* value", L->router_kind);
        return CHRONOS_E_ARG;
    }
    const void* need[] = {L->gu_w, L->gu_s, L->gu_s2, L->gu_beta, L->dn_w, L->dn_s, L->dn_s2, L->dn_beta, L->u_gu, L->v_gu,
                          L->u_dn, L->v_dn_t, L->gu_cin, L->gu_cs2, L->gu_rout, L->gu_rs2, L->dn_cin, L->dn_cs2, L->dn_rout,
                          L->dn_rs2};
    const char* names[] = {"gu_w", "gu_s", "gu_s2", "gu_beta", "dn_w", "dn_s", "dn_s2", "dn_beta", "u_gu", "v_gu",
                           "u_dn", "v_dn_t", "gu_cin", "gu_cs2", "gu_rout", "gu_rs2", "dn_cin", "dn_cs2", "dn_rout",
                           "dn_rs2"};
    // a layer may hold its banks as re-tiled stage images only (gu_t / dn_t): the on-disk-order copies are then optional
    const bool images_only = L->gu_t != nullptr && L->dn_t != nullptr && aligned16(L->gu_t) && aligned16(L->dn_t);
    for (size_t i = 0; i < sizeof(need) / sizeof(need[0]); ++i) {
        const bool scalar_table = (i == 2 || i == 3 || i == 6 || i == 7);
        const bool bank_bytes = (i == 0 || i == 1 || i == 4 || i == 5);
        if (bank_bytes && need[i] == nullptr && images_only) continue;
        if (need[i] == nullptr || (!scalar_table && !aligned16(need[i]))) {
            set_error("layer.%s is NULL or not 16-byte aligned", names[i]);
            return CHRONOS_E_ALIGN;
        }
    }
    if (L->tail_bits != 0) {
        const int gb = L->tail_bits & 0xff, db = (L->tail_bits >> 8) & 0xff;
        if ((gb != 1 && gb != 2) || (db != 1 && db != 2) || (L->tail_bits >> 16) != 0) {
            set_error("tail_bits 0x%x: gate_up and down tail widths must each be 1 or 2", L->tail_bits);
            return CHRONOS_E_ARG;
        }
        const void* tl[] = {L->tail_gu_p, L->tail_gu_s, L->tail_dn_p, L->tail_dn_s};
        for (const void* q : tl)
            if (!aligned16(q)) { set_error("a tail-lattice pointer is NULL or not 16-byte aligned"); return CHRONOS_E_ALIGN; }
    }
    if (need_router && !aligned16(L->router_w)) { set_error("layer.router_w is NULL or not 16-byte aligned"); return CHRONOS_E_ALIGN; }
    if (shared_is_fp8(*L)) {
        if (!aligned16(L->sh8_gu_w) || !aligned16(L->sh8_dn_w) || !L->sh8_gu_s || !L->sh8_dn_s) {
            set_error("a block-FP8 shared-expert pointer is NULL or not 16-byte aligned");
            return CHRONOS_E_ALIGN;
        }
    } else if (L->shared_inter > 0) {
        const void* sh[] = {L->sh_gu_w, L->sh_gu_s, L->sh_dn_w, L->sh_dn_s};
        const bool sh_images_only = aligned16(L->sh_gu_t) && aligned16(L->sh_dn_t);
        for (const void* q : sh)
            if (!aligned16(q) && !(q == nullptr && sh_images_only)) { set_error("a shared-expert bank pointer is NULL or not 16-byte aligned"); return CHRONOS_E_ALIGN; }
        if (!L->sh_gu_s2 || !L->sh_dn_s2) { set_error("a shared-expert scale_2 pointer is NULL"); return CHRONOS_E_ALIGN; }
    }
    return CHRONOS_OK;
}

// The router entry point reads only the router fields, so an expert-parallel shard can route over the full
// (replicated) router table while its bank tables hold the local slots.
static int validate_router(const chronos_layer_t* L) {
    if (!L) { set_error("layer is NULL"); return CHRONOS_E_ALIGN; }
    if (L->hidden <= 0 || L->hidden % 128 || L->hidden > 32768) { set_error("router: hidden (%d) must be a positive multiple of 128", L->hidden); return CHRONOS_E_SHAPE; }
    if (L->n_experts <= 0 || L->n_experts > 1024 || L->top_k <= 0 || L->top_k > kMaxTopK || L->top_k > L->n_experts) {
        set_error("router: n_experts (%d) in [1, 1024] and top_k (%d) in [1, min(%d, n_experts)] required", L->n_experts, L->top_k, kMaxTopK);
        return CHRONOS_E_SHAPE;
    }
    if (L->router_kind < CHRONOS_ROUTER_SOFTMAX_TOPK || L->router_kind > CHRONOS_ROUTER_SQRT_SOFTPLUS) { set_error("router_kind %d is not a CHRONOS_ROUTER_* value", L->router_kind); return CHRONOS_E_ARG; }
    // the router kernels fetch rows with 16-byte bulk copies and vector loads
    if (!aligned16(L->router_w)) { set_error("layer.router_w is NULL or not 16-byte aligned"); return CHRONOS_E_ALIGN; }
    return CHRONOS_OK;
}

static int validate_io(const void* x, int x_dtype, int n_tokens, const void* y, int y_dtype) {
    if (n_tokens < 0 || n_tokens > (1 << 20)) { set_error("n_tokens (%d) out of range", n_tokens); return CHRONOS_E_SHAPE; }
    if ((x_dtype != CHRONOS_DTYPE_F32 && x_dtype != CHRONOS_DTYPE_BF16) ||
        (y_dtype != CHRONOS_DTYPE_F32 && y_dtype != CHRONOS_DTYPE_BF16)) {
        set_error("dtype must be CHRONOS_DTYPE_F32 or CHRONOS_DTYPE_BF16");
        return CHRONOS_E_ARG;
    }
    if (n_tokens > 0 && (!aligned16(x) || !aligned16(y))) { set_error("x or y is NULL or not 16-byte aligned"); return CHRONOS_E_ALIGN; }
    return CHRONOS_OK;
}

// Profiling aid: events recorded between the launches of a forward call (see chronos_b200_set_stage_events).
static thread_local cudaEvent_t g_stage_events[kStageEvents];
static thread_local int g_n_stage_events = 0;

static void stage_mark(int idx, cudaStream_t st) {
    if (idx < g_n_stage_events) cudaEventRecord(g_stage_events[idx], st);
}

// Regime choice when the caller leaves it open: the tensor-core pass pays off once a slot sees enough pairs to
// fill MMA tiles; below that the bank bytes dominate and the streaming pass reads each of them exactly once.
static int pick_regime(const chronos_layer_t& L, int n_tokens, int regime, const Plan& p) {
    if (regime == CHRONOS_REGIME_STREAM_FP4 && !p.fp4_stream) regime = CHRONOS_REGIME_STREAM;  // no re-tiled banks / batch too large
    if (regime == CHRONOS_REGIME_TENSOR_FP4 && !p.fp4_wide) regime = CHRONOS_REGIME_TENSOR;   // no re-tiled banks / batch too small
    if (regime != CHRONOS_REGIME_AUTO) return regime;
    if ((long)n_tokens * L.top_k >= 16L * L.n_slots) return p.fp4_wide ? CHRONOS_REGIME_TENSOR_FP4 : CHRONOS_REGIME_TENSOR;
    return p.fp4_stream ? CHRONOS_REGIME_STREAM_FP4 : CHRONOS_REGIME_STREAM;
}

// Decode-sized batch in the FP4 streaming regime: five launches (csrc/decode_fused.cu). `ids_in` NULL: the front kernel
// routes by itself; otherwise the caller's routing is used and the token scales come from a kernel of their own.
static int fused_decode_forward(const chronos_layer_t& L, const void* x, int x_dtype, int n_tokens, const int32_t* ids_in,
                                const float* gates_in, int shared_first, int shared_count, void* y, int y_dtype, const Plan& plan,
                                cudaStream_t st) {
    Plan p = plan;
    p.gitem_pairs = 8;
    const int with_shared = (shared_count > 0 && shared_is_nvfp4(L)) ? 1 : 0;
    p.shared_lo = with_shared ? shared_first : 0;
    p.shared_n = with_shared ? shared_count : 0;
    // counters, status word and the grid hand-off counter start at zero (a memset node, no allocation)
    if (cudaMemsetAsync(p.counters, 0, 64, st) != cudaSuccess) return check_launch("clear counters");
    if (ids_in != nullptr)
        if (int rc = launch_token_scale(x, x_dtype, n_tokens, L.hidden, p.tok_scale, st)) return rc;
    if (int rc = launch_decode_front(L, x, x_dtype, n_tokens, ids_in, with_shared, p, st)) return rc;
    stage_mark(1, st);
    stage_mark(2, st);
    stage_mark(3, st);
    if (int rc = launch_bank_fp4_fused(L, 0, p, x, x_dtype, st)) return rc;
    stage_mark(4, st);
    if (int rc = launch_decode_mid(L, p, st)) return rc;
    stage_mark(5, st);
    if (int rc = launch_bank_fp4_fused(L, 1, p, x, x_dtype, st)) return rc;
    stage_mark(6, st);
    int rc = launch_decode_combine(L, p, ids_in != nullptr ? ids_in : p.ids, ids_in != nullptr ? gates_in : p.gates, n_tokens, with_shared, y, y_dtype, st);
    if (!rc && shared_is_fp8(L)) rc = launch_shared_fp8(L, x, x_dtype, p, shared_first, shared_count, y, y_dtype, st);
    stage_mark(7, st);
    return rc;
}

static int routed_forward(const chronos_layer_t& L, const void* x, int x_dtype, int n_tokens, const int32_t* ids,
                          const float* gates, int shared_first, int shared_count, void* y, int y_dtype, const Plan& plan,
                          int regime, bool have_tok_scale, const TopkArgs& tk, cudaStream_t st) {
    const int reg = pick_regime(L, n_tokens, regime, plan);
    if ((reg == CHRONOS_REGIME_STREAM || reg == CHRONOS_REGIME_TENSOR) &&
        (L.gu_w == nullptr || L.dn_w == nullptr || (shared_is_nvfp4(L) && L.sh_gu_w == nullptr))) {
        set_error("regime %d reads the banks in their on-disk order, but this layer holds them as FP4 stage images only "
                  "(load it with the on-disk-order copy kept, or use an FP4 regime)", reg);
        return CHRONOS_E_ARG;
    }
    const bool wide = reg == CHRONOS_REGIME_TENSOR_FP4;
    const bool tensor = reg == CHRONOS_REGIME_TENSOR || wide;
    const int fp4 = wide ? 2 : (reg == CHRONOS_REGIME_STREAM_FP4 ? 1 : 0);
    Plan p = plan;
    p.gitem_pairs = wide ? kPairsPerWideItem : kPairsPerGemmItem;
    const int with_shared = (shared_count > 0 && shared_is_nvfp4(L)) ? 1 : 0;
    p.shared_lo = with_shared ? shared_first : 0;
    p.shared_n = with_shared ? shared_count : 0;
    stage_mark(1, st);
    // token scales come from the router kernel when this call ran it; otherwise from a kernel of their own
    if (!have_tok_scale)
        if (int rc = launch_token_scale(x, x_dtype, n_tokens, L.hidden, p.tok_scale, st)) return rc;
    if (int rc = launch_plan(L, ids, n_tokens, with_shared, have_tok_scale ? 0 : 1, tk, p, st)) return rc;
    stage_mark(2, st);
    // many pairs per expert (the batch shapes the tensor regime is chosen for): healer products on the tensor cores when
    // the layer carries healer.v_down in its on-disk orientation, else CUDA-core kernels that share healer rows through L1
    const int many = (tensor && p.yt != nullptr) ? 1 : 0;
    const bool hmma = many && healer_mma_fits(L);
    const bool tail = p.tail_gu != nullptr;
    if (hmma || tail)  // the large-batch kernels and the tail pass read a token's row once per pair: give them x / token scale as fp16
        if (int rc = launch_tokens_f16(x, x_dtype, n_tokens, L.hidden, p.tok_scale, p.x16, st)) return rc;
    if (int rc = launch_pre_gu(L, x, x_dtype, p, fp4, hmma ? 2 : many, st)) return rc;
    if (hmma)
        if (int rc = launch_healer_in_mma(L, 0, p.x16, kDtypeF16Scaled, p, st)) return rc;
    if (hmma && wide && healer_fused(L, p))  // the healer factors as an operand tile: the bank pass adds the correction itself
        if (int rc = launch_heal_image(L, 0, p, st)) return rc;
    if (tail)
        if (int rc = launch_tail_pass(L, 0, p.x16, kDtypeF16Scaled, p, st)) return rc;
    stage_mark(3, st);
    if (int rc = wide ? launch_bank_fp4_wide(L, 0, p, st)
                      : (tensor ? launch_bank_gemm(L, 0, p, st) : (fp4 ? launch_bank_fp4(L, 0, p, st) : launch_bank_stream(L, 0, p, st)))) return rc;
    stage_mark(4, st);
    if (int rc = hmma ? launch_mid_mma(L, p, wide ? 1 : 0, st) : launch_mid(L, p, fp4, st)) return rc;
    if (tail)  // SwiGLU outputs in natural order: fp16 rows / pair scale in the FP4 tensor regime, fp32 rows otherwise
        if (int rc = wide ? launch_tail_pass(L, 1, p.ac, kDtypeF16Scaled, p, st) : launch_tail_pass(L, 1, p.act, CHRONOS_DTYPE_F32, p, st)) return rc;
    stage_mark(5, st);
    if (int rc = wide ? launch_bank_fp4_wide(L, 1, p, st)
                      : (tensor ? launch_bank_gemm(L, 1, p, st) : (fp4 ? launch_bank_fp4(L, 1, p, st) : launch_bank_stream(L, 1, p, st)))) return rc;
    stage_mark(6, st);
    int rc;
    if (hmma && wide && healer_fused(L, p)) {
        // the down pass already added the healer term: one kernel gathers the token's rows and sums them
        rc = launch_combine_gather(L, p, gates, n_tokens, with_shared, y, y_dtype, st);
    } else if (hmma) {
        rc = launch_down_out_mma(L, p, st);
        if (!rc) rc = launch_combine_sum(L, p, gates, n_tokens, with_shared, y, y_dtype, st);
    } else {
        rc = many ? launch_combine_tiled(L, p, gates, n_tokens, with_shared, y, y_dtype, st)
                  : launch_combine(L, p, gates, n_tokens, with_shared, y, y_dtype, st);
    }
    if (!rc && shared_is_fp8(L)) rc = launch_shared_fp8(L, x, x_dtype, p, shared_first, shared_count, y, y_dtype, st);
    stage_mark(7, st);
    return rc;
}

}  // namespace chronos

using namespace chronos;

extern "C" {

int chronos_b200_abi_version(void) { return 11; }

const char* chronos_b200_last_error(void) { return g_err; }

int chronos_b200_dequant_nvfp4(const uint8_t* packed, const uint8_t* scale, const float* scale_2, float* out, int rows,
                               int cols, void* stream) {
    if (rows <= 0 || cols <= 0 || cols % 16) { set_error("dequant: rows (%d) > 0 and cols (%d) a positive multiple of 16 required", rows, cols); return CHRONOS_E_SHAPE; }
    if (!packed || !scale || !scale_2 || !out || (reinterpret_cast<uintptr_t>(out) & 7u)) { set_error("dequant: NULL or misaligned pointer"); return CHRONOS_E_ALIGN; }
    return launch_dequant(packed, scale, scale_2, out, rows, cols, (cudaStream_t)stream);
}

int chronos_b200_dequant_fp8_block(const uint8_t* w, const float* scale_inv, float* out, int rows, int cols, void* stream) {
    if (rows <= 0 || cols <= 0) { set_error("dequant_fp8_block: rows (%d) and cols (%d) must be positive", rows, cols); return CHRONOS_E_SHAPE; }
    if (!w || !scale_inv || !out) { set_error("dequant_fp8_block: NULL pointer"); return CHRONOS_E_ALIGN; }
    return launch_dequant_fp8_block(w, scale_inv, out, rows, cols, (cudaStream_t)stream);
}

int chronos_b200_unfold_expert_fp32(const chronos_layer_t* layer, int expert, int which, float* out, float* scratch,
                                    void* stream) {
    if (int rc = validate_layer(layer, false)) return rc;
    if (expert < 0 || expert >= layer->n_experts || (which != 0 && which != 1)) { set_error("unfold: expert %d / which %d out of range", expert, which); return CHRONOS_E_ARG; }
    if (!out || !scratch) { set_error("unfold: out or scratch is NULL"); return CHRONOS_E_ALIGN; }
    if (!layer->gu_w || !layer->dn_w) { set_error("unfold: the layer holds no on-disk-order banks (FP4 stage images only)"); return CHRONOS_E_ARG; }
    if (int rc = launch_unfold(*layer, expert, which, out, scratch, (cudaStream_t)stream)) return rc;
    return layer->tail_bits ? launch_tail_add(*layer, expert, which, out, (cudaStream_t)stream) : CHRONOS_OK;
}

int chronos_b200_unfold_expert_fp32_static(const chronos_layer_t* layer, int expert, int which, float* out, void* stream) {
    if (int rc = validate_layer(layer, false)) return rc;
    if (expert < 0 || expert >= layer->n_experts || (which != 0 && which != 1)) { set_error("unfold_static: expert %d / which %d out of range", expert, which); return CHRONOS_E_ARG; }
    if (!out) { set_error("unfold_static: out is NULL"); return CHRONOS_E_ALIGN; }
    if (!layer->gu_w || !layer->dn_w) { set_error("unfold_static: the layer holds no on-disk-order banks (FP4 stage images only)"); return CHRONOS_E_ARG; }
    if (int rc = launch_unfold_static(*layer, expert, which, out, (cudaStream_t)stream)) return rc;
    return layer->tail_bits ? launch_tail_add(*layer, expert, which, out, (cudaStream_t)stream) : CHRONOS_OK;
}

int chronos_b200_router_topk(const chronos_layer_t* layer, const void* x, int x_dtype, int n_tokens, int32_t* ids,
                             float* gates, float* logits, void* stream) {
    if (int rc = validate_router(layer)) return rc;
    if (int rc = validate_io(x, x_dtype, n_tokens, x, CHRONOS_DTYPE_F32)) return rc;
    if (!ids || !gates || !logits) { set_error("router: ids, gates or logits is NULL"); return CHRONOS_E_ALIGN; }
    return launch_router(*layer, x, x_dtype, n_tokens, ids, gates, logits, nullptr, nullptr, (cudaStream_t)stream);
}

int chronos_b200_router_topk_coalesced(const chronos_layer_t* layer, const void* x, int x_dtype, int n_tokens, int tokens_per_stream,
                                       int pool, int keep, float bonus, int32_t* ids, float* gates, float* logits, void* stream) {
    if (int rc = validate_router(layer)) return rc;
    if (int rc = validate_io(x, x_dtype, n_tokens, x, CHRONOS_DTYPE_F32)) return rc;
    if (!ids || !gates || !logits) { set_error("router_coalesced: ids, gates or logits is NULL"); return CHRONOS_E_ALIGN; }
    if (tokens_per_stream < 1 || pool < layer->top_k || pool > 32 || pool > layer->n_experts || keep < 0 || keep > layer->top_k || !(bonus >= 0.0f)) {
        set_error("router_coalesced: tokens_per_stream (%d) >= 1, top_k <= pool (%d) <= min(32, n_experts), 0 <= keep (%d) <= top_k and bonus >= 0 required",
                  tokens_per_stream, pool, keep);
        return CHRONOS_E_ARG;
    }
    if (n_tokens == 0) return CHRONOS_OK;
    // logits exactly as the plain router computes them (ids == NULL: no top-k there), then the coalescing selection
    if (int rc = launch_router(*layer, x, x_dtype, n_tokens, nullptr, gates, logits, nullptr, nullptr, (cudaStream_t)stream)) return rc;
    return launch_coalesced_topk(*layer, logits, n_tokens, tokens_per_stream, pool, keep, bonus, ids, gates, (cudaStream_t)stream);
}

size_t chronos_b200_workspace_bytes(const chronos_layer_t* layer, int n_tokens) {
    if (validate_layer(layer, false) != CHRONOS_OK || n_tokens < 0 || n_tokens > (1 << 20)) return 0;
    return plan_layout(*layer, n_tokens).total;
}

long chronos_b200_workspace_status_offset(const chronos_layer_t* layer, int n_tokens) {
    if (validate_layer(layer, false) != CHRONOS_OK || n_tokens < 0 || n_tokens > (1 << 20)) return -1;
    return (long)plan_layout(*layer, n_tokens).off_counters + 2 * (long)sizeof(int32_t);
}

static int full_forward(const chronos_layer_t* layer, const void* x, int x_dtype, int n_tokens, void* y, int y_dtype,
                        void* workspace, size_t workspace_bytes, int regime, void* stream) {
    if (int rc = validate_layer(layer, true)) return rc;
    if (int rc = validate_io(x, x_dtype, n_tokens, y, y_dtype)) return rc;
    if (regime < CHRONOS_REGIME_AUTO || regime > CHRONOS_REGIME_TENSOR_FP4) { set_error("regime %d is not a CHRONOS_REGIME_* value", regime); return CHRONOS_E_ARG; }
    if (n_tokens == 0) return CHRONOS_OK;
    const PlanLayout lay = plan_layout(*layer, n_tokens);
    if (!aligned16(workspace) || workspace_bytes < lay.total) {
        set_error("workspace of %zu bytes is too small or misaligned (%zu needed)", workspace_bytes, lay.total);
        return CHRONOS_E_WORKSPACE;
    }
    const Plan p = plan_bind(lay, workspace);
    cudaStream_t st = (cudaStream_t)stream;
    stage_mark(0, st);
    if (pick_regime(*layer, n_tokens, regime, p) == CHRONOS_REGIME_STREAM_FP4 && decode_fused_fits(*layer, x_dtype, n_tokens, p))
        return fused_decode_forward(*layer, x, x_dtype, n_tokens, nullptr, nullptr, 0, n_tokens, y, y_dtype, p, st);
    // the router may raise the status word, so it is cleared here (a memset node, no allocation) and not by the plan kernel
    if (cudaMemsetAsync(p.counters, 0, 64, st) != cudaSuccess) return check_launch("clear counters");
    // decode-sized batches: the top-k runs inside the plan launch (one launch less on the critical path)
    const bool fuse_topk = n_tokens <= 32;
    TopkArgs tk{};
    if (fuse_topk)
        tk = TopkArgs{p.logits, layer->e_bias, layer->router_kind, layer->renorm, layer->routed_scaling, n_tokens,
                      layer->n_experts, layer->top_k, p.ids, p.gates};
    if (int rc = launch_router(*layer, x, x_dtype, n_tokens, fuse_topk ? nullptr : p.ids, p.gates, p.logits, p.tok_scale,
                               p.counters + 2, st))
        return rc;
    return routed_forward(*layer, x, x_dtype, n_tokens, p.ids, p.gates, 0, n_tokens, y, y_dtype, p, regime, true, tk, st);
}

int chronos_b200_folded_moe_decode(const chronos_layer_t* layer, const void* x, int x_dtype, int n_tokens, void* y,
                                   int y_dtype, void* workspace, size_t workspace_bytes, void* stream) {
    return full_forward(layer, x, x_dtype, n_tokens, y, y_dtype, workspace, workspace_bytes, CHRONOS_REGIME_STREAM_FP4, stream);
}

int chronos_b200_folded_moe_prefill(const chronos_layer_t* layer, const void* x, int x_dtype, int n_tokens, void* y,
                                    int y_dtype, void* workspace, size_t workspace_bytes, void* stream) {
    return full_forward(layer, x, x_dtype, n_tokens, y, y_dtype, workspace, workspace_bytes, CHRONOS_REGIME_TENSOR_FP4, stream);
}

int chronos_b200_folded_moe_forward(const chronos_layer_t* layer, const void* x, int x_dtype, int n_tokens, void* y,
                                    int y_dtype, void* workspace, size_t workspace_bytes, void* stream) {
    return full_forward(layer, x, x_dtype, n_tokens, y, y_dtype, workspace, workspace_bytes, CHRONOS_REGIME_AUTO, stream);
}

int chronos_b200_folded_moe_routed(const chronos_layer_t* layer, const void* x, int x_dtype, int n_tokens,
                                   const int32_t* ids, const float* gates, int shared_first, int shared_count, int regime,
                                   void* y, int y_dtype, void* workspace, size_t workspace_bytes, void* stream) {
    if (int rc = validate_layer(layer, false)) return rc;
    if (regime < CHRONOS_REGIME_AUTO || regime > CHRONOS_REGIME_TENSOR_FP4) { set_error("regime %d is not a CHRONOS_REGIME_* value", regime); return CHRONOS_E_ARG; }
    if (int rc = validate_io(x, x_dtype, n_tokens, y, y_dtype)) return rc;
    if (n_tokens == 0) return CHRONOS_OK;
    if (!ids || !gates) { set_error("routed: ids or gates is NULL"); return CHRONOS_E_ALIGN; }
    if (shared_count < 0 || shared_first < 0 || (long)shared_first + shared_count > n_tokens) {
        set_error("routed: shared-expert token range [%d, %d + %d) does not lie inside the %d tokens", shared_first, shared_first, shared_count, n_tokens);
        return CHRONOS_E_ARG;
    }
    const PlanLayout lay = plan_layout(*layer, n_tokens);
    if (!aligned16(workspace) || workspace_bytes < lay.total) {
        set_error("workspace of %zu bytes is too small or misaligned (%zu needed)", workspace_bytes, lay.total);
        return CHRONOS_E_WORKSPACE;
    }
    const Plan p = plan_bind(lay, workspace);
    if (pick_regime(*layer, n_tokens, regime, p) == CHRONOS_REGIME_STREAM_FP4 && decode_fused_fits(*layer, x_dtype, n_tokens, p)) {
        stage_mark(1, (cudaStream_t)stream);
        return fused_decode_forward(*layer, x, x_dtype, n_tokens, ids, gates, shared_first, shared_count, y, y_dtype, p, (cudaStream_t)stream);
    }
    return routed_forward(*layer, x, x_dtype, n_tokens, ids, gates, shared_first, shared_count, y, y_dtype, p, regime, false, TopkArgs{}, (cudaStream_t)stream);
}

int chronos_b200_fp4_mma_probe(const uint8_t* a_image, const uint8_t* b_image, int n_stages, int b_rows, float* d_out,
                               int32_t* status, void* stream) {
    if (n_stages <= 0 || n_stages > 4096) { set_error("fp4_probe: n_stages (%d) out of range", n_stages); return CHRONOS_E_SHAPE; }
    if (b_rows < 16 || b_rows > 256 || b_rows % 16) { set_error("fp4_probe: b_rows (%d) must be a multiple of 16 in 16..256", b_rows); return CHRONOS_E_SHAPE; }
    if (!aligned16(a_image) || !aligned16(b_image) || !d_out || !status) { set_error("fp4_probe: NULL or misaligned pointer"); return CHRONOS_E_ALIGN; }
    return launch_fp4_probe(a_image, b_image, n_stages, b_rows, d_out, status, (cudaStream_t)stream);
}

static int validate_ep(int n_tokens, int top_k, int hidden, int world, int capacity) {
    if (n_tokens < 0 || n_tokens > (1 << 20) || top_k <= 0 || top_k > kMaxTopK || hidden <= 0 || hidden % 8 || world <= 0 || world > 64 ||
        capacity <= 0 || capacity > (1 << 20)) {
        set_error("ep: n_tokens %d, top_k %d, hidden %d (multiple of 8), world %d (<= 64) or capacity %d out of range", n_tokens, top_k, hidden, world, capacity);
        return CHRONOS_E_SHAPE;
    }
    return CHRONOS_OK;
}

int chronos_b200_ep_pack(const void* x, int x_dtype, const int32_t* ids, const float* gates, int n_tokens, int top_k, int hidden,
                         int world, int experts_per_rank, int capacity, void* send_rows, int32_t* send_meta, int32_t* slot_of,
                         int32_t* overflow, int block_rows, long meta_block_ints, void* stream) {
    if (int rc = validate_ep(n_tokens, top_k, hidden, world, capacity)) return rc;
    if (x_dtype != CHRONOS_DTYPE_F32 && x_dtype != CHRONOS_DTYPE_BF16) { set_error("ep_pack: bad dtype"); return CHRONOS_E_ARG; }
    if (experts_per_rank <= 0) { set_error("ep_pack: experts_per_rank (%d) must be positive", experts_per_rank); return CHRONOS_E_SHAPE; }
    if (n_tokens > 0 && (!aligned16(x) || !aligned16(send_rows) || !ids || !gates || !send_meta || !slot_of || !overflow)) {
        set_error("ep_pack: NULL or misaligned pointer");
        return CHRONOS_E_ALIGN;
    }
    if ((block_rows != 0 && block_rows < capacity) || (meta_block_ints != 0 && meta_block_ints < (long)(capacity + 1) * (2 * top_k + 2))) {
        set_error("ep_pack: block strides (%d rows, %ld words) smaller than a block", block_rows, meta_block_ints);
        return CHRONOS_E_SHAPE;
    }
    return launch_ep_pack(x, x_dtype, ids, gates, n_tokens, top_k, hidden, world, experts_per_rank, capacity, send_rows, send_meta, slot_of,
                          overflow, block_rows, meta_block_ints, (cudaStream_t)stream);
}

int chronos_b200_ep_pack_peer(const void* x, int x_dtype, const int32_t* ids, const float* gates, int n_tokens, int top_k, int hidden,
                              int world, int experts_per_rank, int capacity, void* const* peer_bases, int my_rank, int block_rows,
                              int32_t* slot_of, int32_t* overflow, void* stream) {
    if (int rc = validate_ep(n_tokens, top_k, hidden, world, capacity)) return rc;
    if (x_dtype != CHRONOS_DTYPE_F32 && x_dtype != CHRONOS_DTYPE_BF16) { set_error("ep_pack_peer: bad dtype"); return CHRONOS_E_ARG; }
    if (experts_per_rank <= 0 || my_rank < 0 || my_rank >= world) { set_error("ep_pack_peer: bad rank / experts_per_rank"); return CHRONOS_E_SHAPE; }
    const long meta_bytes = (long)(capacity + 1) * (2 * top_k + 2) * 4, row_bytes = (long)hidden * (x_dtype == CHRONOS_DTYPE_BF16 ? 2 : 4);
    if ((long)(block_rows - capacity) * row_bytes < meta_bytes) {
        set_error("ep_pack_peer: block_rows (%d) leaves no room for %ld bytes of metadata behind %d rows", block_rows, meta_bytes, capacity);
        return CHRONOS_E_SHAPE;
    }
    if (n_tokens > 0 && (!aligned16(x) || !peer_bases || !ids || !gates || !slot_of || !overflow)) {
        set_error("ep_pack_peer: NULL or misaligned pointer");
        return CHRONOS_E_ALIGN;
    }
    return launch_ep_pack_peer(x, x_dtype, ids, gates, n_tokens, top_k, hidden, world, experts_per_rank, capacity, peer_bases, my_rank,
                               block_rows, slot_of, overflow, (cudaStream_t)stream);
}

int chronos_b200_ep_send_back_peer(const void* part_rows, int dtype, int hidden, int world, int block_rows, int capacity, int top_k,
                                   const void* recv_base, void* const* peer_back, int my_rank, void* stream) {
    if (int rc = validate_ep(0, top_k, hidden, world, capacity)) return rc;
    if (dtype != CHRONOS_DTYPE_F32 && dtype != CHRONOS_DTYPE_BF16) { set_error("ep_send_back_peer: bad dtype"); return CHRONOS_E_ARG; }
    if (block_rows < capacity || my_rank < 0 || my_rank >= world) { set_error("ep_send_back_peer: bad block_rows / rank"); return CHRONOS_E_SHAPE; }
    if (!aligned16(part_rows) || !aligned16(recv_base) || !peer_back) { set_error("ep_send_back_peer: NULL or misaligned pointer"); return CHRONOS_E_ALIGN; }
    return launch_ep_send_back_peer(part_rows, dtype, hidden, world, block_rows, capacity, top_k, recv_base, peer_back, my_rank, (cudaStream_t)stream);
}

int chronos_b200_ep_barrier(void* const* pads, int my_rank, int world, uint32_t epoch, int32_t* status, void* stream) {
    if (!pads || !status || world < 1 || world > 1024 || my_rank < 0 || my_rank >= world) {
        set_error("ep_barrier: bad arguments (world %d, rank %d)", world, my_rank);
        return CHRONOS_E_ARG;
    }
    return launch_ep_barrier(pads, my_rank, world, epoch, status, (cudaStream_t)stream);
}

int chronos_b200_ep_unpack_meta(const int32_t* recv_meta, int world, int capacity, int top_k, int32_t* ids_out, float* gates_out,
                                int block_rows, long meta_block_ints, int tail_rows, void* stream) {
    if (int rc = validate_ep(0, top_k, 8, world, capacity)) return rc;
    if (!recv_meta || !ids_out || !gates_out) { set_error("ep_unpack_meta: NULL pointer"); return CHRONOS_E_ALIGN; }
    if ((block_rows != 0 && block_rows < capacity) || tail_rows < 0 ||
        (meta_block_ints != 0 && meta_block_ints < (long)(capacity + 1) * (2 * top_k + 2))) {
        set_error("ep_unpack_meta: block strides (%d rows, %ld words) smaller than a block, or negative tail", block_rows, meta_block_ints);
        return CHRONOS_E_SHAPE;
    }
    return launch_ep_unpack_meta(recv_meta, world, capacity, top_k, ids_out, gates_out, block_rows, meta_block_ints, tail_rows, (cudaStream_t)stream);
}

int chronos_b200_ep_combine(const void* back_rows, int dtype, const int32_t* slot_of, const void* extra, int n_tokens, int hidden, int world,
                            int capacity, void* y, int y_dtype, int block_rows, void* stream) {
    if (int rc = validate_ep(n_tokens, 1, hidden, world, capacity)) return rc;
    if ((dtype != CHRONOS_DTYPE_F32 && dtype != CHRONOS_DTYPE_BF16) || (y_dtype != CHRONOS_DTYPE_F32 && y_dtype != CHRONOS_DTYPE_BF16)) {
        set_error("ep_combine: bad dtype");
        return CHRONOS_E_ARG;
    }
    if (n_tokens > 0 && (!aligned16(back_rows) || !aligned16(y) || !slot_of || (extra != nullptr && !aligned16(extra)))) {
        set_error("ep_combine: NULL or misaligned pointer");
        return CHRONOS_E_ALIGN;
    }
    if (block_rows != 0 && block_rows < capacity) { set_error("ep_combine: block stride (%d rows) smaller than a block", block_rows); return CHRONOS_E_SHAPE; }
    return launch_ep_combine(back_rows, dtype, slot_of, extra, n_tokens, hidden, world, capacity, y, y_dtype, block_rows, (cudaStream_t)stream);
}

int chronos_b200_wait_probe(int32_t* status, unsigned poll_limit, void* stream) {
    if (!status) { set_error("wait_probe: status is NULL"); return CHRONOS_E_ALIGN; }
    if (poll_limit == 0 || poll_limit > 4096) { set_error("wait_probe: poll_limit (%u) must be in 1..4096", poll_limit); return CHRONOS_E_ARG; }
    return launch_wait_probe(status, poll_limit, (cudaStream_t)stream);
}

int chronos_b200_set_stage_events(void** events, int n_events) {
    if (n_events < 0 || n_events > kStageEvents || (n_events > 0 && !events)) { set_error("set_stage_events: 0..%d events expected", kStageEvents); return CHRONOS_E_ARG; }
    for (int i = 0; i < n_events; ++i) g_stage_events[i] = (cudaEvent_t)events[i];
    g_n_stage_events = n_events;
    return CHRONOS_OK;
}

int chronos_b200_residual_rmsnorm(void* h, const void* y, const float* weight, void* x_norm, int dtype, int n_tokens,
                                  int hidden, float eps, void* stream) {
    if (dtype != CHRONOS_DTYPE_F32 && dtype != CHRONOS_DTYPE_BF16) { set_error("rmsnorm: bad dtype"); return CHRONOS_E_ARG; }
    if (n_tokens < 0 || hidden <= 0) { set_error("rmsnorm: bad shape"); return CHRONOS_E_SHAPE; }
    if (n_tokens > 0 && (!h || !x_norm)) { set_error("rmsnorm: NULL pointer"); return CHRONOS_E_ALIGN; }
    return launch_residual_rmsnorm(h, y, weight, x_norm, dtype, n_tokens, hidden, eps, (cudaStream_t)stream);
}

}  // extern "C"
