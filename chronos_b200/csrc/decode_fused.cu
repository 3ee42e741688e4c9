// Fused decode path of the FP4 streaming regime: the kernels around the two bank passes, cut so that a decode step is
// five launches whose small ones do no healer work at all.
//
//   decode_front_kernel   router logits -> (grid-wide hand-off) -> top-k + batch coalescing, done by EVERY CTA for itself
//                         in shared memory (the result is deterministic, so all CTAs agree; CTA 0 publishes it) ->
//                         gate_up input transform into the FP4 activation images
//   bank pass (gate_up)   bank_fp4_kernel; its side warps compute the healer term U_gu (V_gu x) meanwhile (mma.sync)
//   decode_mid_kernel     one CTA per pair: inverse-row gather, beta, + healer term, SwiGLU, pair scale, down-input
//                         transform into the FP4 image
//   bank pass (down)      bank_fp4_kernel; its side warps compute U_down (V_down act) meanwhile
//   decode_combine_kernel inverse-row gather, beta, + healer term, gate-weighted sum over the token's experts (+ shared)
//
// Mathematics as in csrc/transform_kernels.cu (ChronosGlm5HolographicExpertGroup.forward_cold_fast,
// chronos_1t/models/glm5_chronos_moe.py:149-195); routing as chronos_1t/models/glm53_chronos_moe.py:392-399, :456-459.
#include "common.cuh"

namespace chronos {

constexpr int kFrontThreads = 512;
constexpr int kFrontWarps = kFrontThreads / 32;
constexpr int kFrontMaxTokens = 32;   // decode-sized batches only
constexpr int kFrontEpc = 2;          // router rows staged per logits tile
constexpr int kFrontBins = 1024 + 2;  // experts + shared-expert bin + total
constexpr int kFrontMaxPairs = kFrontMaxTokens * kMaxTopK + kFrontMaxTokens;
constexpr int kFrontMaxChunks = 1024 + 1 + kFrontMaxPairs / 8 + 1;
constexpr uint32_t kGridWaitLimit = 1u << 21;  // polls of ~0.3 us: well under a second

struct FrontArgs {
    chronos_layer_t L;
    Plan p;
    const void* x;
    int x_dtype, n_tokens;
    const int32_t* ids_in;  // caller-supplied routing (the router phase is skipped and the token scales are ready) or NULL
    const float* gates_in;
    int with_shared;
    int tg;                 // token rows staged per logits tile
};

// Plan of the batch in shared memory (every CTA holds its own, identical copy).
struct FrontPlan {
    int cnt[kFrontBins], off[kFrontBins], cur[kFrontBins], tmp[kFrontBins];
    int ids[kFrontMaxTokens * kMaxTopK];
    float gates[kFrontMaxTokens * kMaxTopK];
    int pair_token[kFrontMaxPairs], pair_expert[kFrontMaxPairs], pair_item[kFrontMaxPairs], pair_pos[kFrontMaxPairs];
    int chunk_start[kFrontMaxChunks], chunk_cnt[kFrontMaxChunks];
    int warp_tot[kFrontWarps + 1];
    int n_pairs, n_items, n_chunks, ok;
};

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// All CTAs of the grid wait here for each other (the launch is cooperative, so they are all resident). Bounded: a CTA
// that gives up raises the status word and the kernel returns.
__device__ __forceinline__ bool grid_hand_off(int32_t* arrivals, int32_t* status, int* ok_s) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(arrivals, 1);
        int ok = 0;
        for (uint32_t it = 0; it < kGridWaitLimit; ++it) {
            int seen;
            asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(seen) : "l"(arrivals) : "memory");
            if (seen >= (int)gridDim.x) { ok = 1; break; }
            __nanosleep(64);
        }
        if (!ok) atomicOr(status, kStatusGridSyncTimeout);
        *ok_s = ok;
    }
    __syncthreads();
    return *ok_s != 0;
}

// In-place exclusive scan of a[0 .. n), n <= kFrontBins - 1, by the whole CTA; a[n] receives the total. Every thread
// owns up to three consecutive elements; warp shuffles inside the warps, then the 16 warp totals. Ends with a barrier.
__device__ __forceinline__ void block_exclusive_scan(int* a, int n, int* warp_tot /*[kFrontWarps + 1]*/) {
    constexpr int PER = (kFrontBins + kFrontThreads - 1) / kFrontThreads;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int v[PER], sum = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int idx = tid * PER + i;
        v[i] = idx < n ? a[idx] : 0;
        sum += v[i];
    }
    int inc = sum;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, inc, d);
        if (lane >= d) inc += o;
    }
    if (lane == 31) warp_tot[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        const int w = lane < kFrontWarps ? warp_tot[lane] : 0;
        int winc = w;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, winc, d);
            if (lane >= d) winc += o;
        }
        if (lane < kFrontWarps) warp_tot[lane] = winc - w;
        if (lane == kFrontWarps - 1) warp_tot[kFrontWarps] = winc;
    }
    __syncthreads();
    int run = warp_tot[warp] + inc - sum;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int idx = tid * PER + i;
        if (idx < n) a[idx] = run;
        run += v[i];
    }
    if (tid == 0) a[n] = warp_tot[kFrontWarps];
    __syncthreads();
}

// Router logits of the tiles this CTA owns, in the stated order (lane l sums k = 128 j + 4 l + i by FMA from +0, j then i
// ascending; xor butterfly 16..1): same bits as router_logits_kernel and as the CPU oracle.
template <bool BF16>
__device__ bool front_logits(const FrontArgs& a, uint8_t* sm, uint64_t* bar) {
    constexpr int XB = BF16 ? 2 : 4;
    const int H = a.L.hidden, E = a.L.n_experts, T = a.n_tokens, tg = a.tg;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int e_tiles = (E + kFrontEpc - 1) / kFrontEpc, t_tiles = (T + tg - 1) / tg;
    float* ws = reinterpret_cast<float*>(sm);
    uint8_t* xs = sm + (size_t)kFrontEpc * H * 4;
    uint32_t phase = 0;
    for (int tile = blockIdx.x; tile < e_tiles * t_tiles; tile += gridDim.x, phase ^= 1u) {
        const int tt = tile / e_tiles, et = tile % e_tiles;
        const int t0 = tt * tg, e0 = et * kFrontEpc;
        const int nt = min(tg, T - t0), ne = min(kFrontEpc, E - e0);
        if (threadIdx.x == 0) {
            mbar_expect_tx(smem_u32(bar), (uint32_t)(ne * H * 4 + nt * H * XB));
            for (int i = 0; i < ne; ++i)
                bulk_g2s(smem_u32(ws + (size_t)i * H), a.L.router_w + (size_t)(e0 + i) * H, (uint32_t)H * 4, smem_u32(bar));
            for (int t = 0; t < nt; ++t)
                bulk_g2s(smem_u32(xs + (size_t)t * H * XB), reinterpret_cast<const uint8_t*>(a.x) + (size_t)(t0 + t) * H * XB,
                         (uint32_t)H * XB, smem_u32(bar));
        }
        const bool ok = mbar_wait(smem_u32(bar), phase);
        if (__syncthreads_or(!ok)) {
            if (threadIdx.x == 0) atomicOr(a.p.counters + 2, kStatusRouterTimeout);
            return false;
        }
        for (int u = warp; u < ne * nt; u += kFrontWarps) {
            const int ew = u / nt, tk = u % nt;
            const float* wr = ws + (size_t)ew * H + 4 * lane;
            float acc = 0.0f, ssq = 0.0f;
            for (int k = 0; k < H; k += 128) {
                const float4 wq = *reinterpret_cast<const float4*>(wr + k);
                float4 xq;
                if (BF16) {
                    const uint2 v = *reinterpret_cast<const uint2*>(xs + ((size_t)tk * H + k + 4 * lane) * 2);
                    xq = make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u), __uint_as_float(v.y << 16),
                                     __uint_as_float(v.y & 0xffff0000u));
                } else {
                    xq = *reinterpret_cast<const float4*>(xs + ((size_t)tk * H + k + 4 * lane) * 4);
                }
                acc = __fmaf_rn(xq.x, wq.x, acc);
                acc = __fmaf_rn(xq.y, wq.y, acc);
                acc = __fmaf_rn(xq.z, wq.z, acc);
                acc = __fmaf_rn(xq.w, wq.w, acc);
                ssq = fmaf(xq.x, xq.x, fmaf(xq.y, xq.y, fmaf(xq.z, xq.z, fmaf(xq.w, xq.w, ssq))));
            }
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
            if (lane == 0) a.p.logits[(size_t)(t0 + tk) * E + e0 + ew] = acc;
            if (e0 + ew == 0) {  // the warp that owns expert 0 of a token also produces the token's power-of-two scale
#pragma unroll
                for (int off = 16; off >= 1; off >>= 1) ssq += __shfl_xor_sync(0xffffffffu, ssq, off);
                if (lane == 0) a.p.tok_scale[t0 + tk] = pow2_scale(ssq, H);
            }
        }
        __syncthreads();  // the staging area is overwritten by the next tile
    }
    return true;
}

// Batch coalescing in shared memory: counting sort of the routing entries by expert (position inside an expert =
// order of (token, entry)), work items of up to 8 pairs per slot, chunks of up to 8 pairs per expert.
__device__ void front_plan(const FrontArgs& a, FrontPlan& s) {
    const int tid = threadIdx.x;
    const int T = a.n_tokens, k = a.L.top_k, E = a.L.n_experts, K = a.L.group_size, n_slots = a.L.n_slots;
    const int n_bins = E + 1, n_entries = T * k;
    const bool pub = blockIdx.x == 0;  // CTA 0 publishes the plan for the kernels that follow
    for (int i = tid; i <= n_bins; i += kFrontThreads) { s.cnt[i] = 0; s.cur[i] = 0; }
    for (int i = tid; i < n_entries; i += kFrontThreads) {  // s.ids holds the routing; anything outside [0, E) is skipped
        const int e = s.ids[i];
        s.ids[i] = (e >= 0 && e < E) ? e : -1;
    }
    __syncthreads();
    for (int i = tid; i < n_entries; i += kFrontThreads)
        if (s.ids[i] >= 0) atomicAdd(&s.cnt[s.ids[i]], 1);
    if (tid == 0 && a.with_shared) s.cnt[E] = a.p.shared_n;
    __syncthreads();
    for (int i = tid; i <= n_bins; i += kFrontThreads) s.off[i] = s.cnt[i];
    __syncthreads();
    block_exclusive_scan(s.off, n_bins, s.warp_tot);
    // position of entry i inside its expert = number of earlier entries (in (token, entry) order) that name the same expert:
    // deterministic, so every CTA builds the same plan
    for (int i = tid; i < n_entries; i += kFrontThreads) {
        const int e = s.ids[i];
        int pos = -1;
        if (e >= 0) {
            int before = 0;
            for (int j = 0; j < i; ++j) before += s.ids[j] == e;
            pos = s.off[e] + before;
            s.pair_token[pos] = i / k;
            s.pair_expert[pos] = e;
        }
        if (pub) a.p.pos_of[i] = pos;
    }
    if (a.with_shared)
        for (int t = tid; t < a.p.shared_n; t += kFrontThreads) {
            s.pair_token[s.off[E] + t] = a.p.shared_lo + t;
            s.pair_expert[s.off[E] + t] = E;
        }
    // streaming work items: slot sl owns sorted pairs [off[sl*K], off[(sl+1)*K]); the shared expert is slot n_slots
    const int n_vslots = n_slots + 1;
    for (int sl = tid; sl < n_vslots; sl += kFrontThreads) {
        const int lo = sl < n_slots ? s.off[sl * K] : s.off[E], hi = sl < n_slots ? s.off[(sl + 1) * K] : s.off[n_bins];
        s.tmp[sl] = (hi - lo + kPairsPerItem - 1) / kPairsPerItem;
    }
    __syncthreads();
    block_exclusive_scan(s.tmp, n_vslots, s.warp_tot);
    for (int sl = tid; sl < n_vslots; sl += kFrontThreads) {
        const int lo = sl < n_slots ? s.off[sl * K] : s.off[E], hi = sl < n_slots ? s.off[(sl + 1) * K] : s.off[n_bins];
        const int first = s.tmp[sl];
        for (int q = 0, at = lo; at < hi; ++q, at += kPairsPerItem) {
            const int it = first + q, c = min(kPairsPerItem, hi - at);
            if (pub && it < a.p.max_items) { a.p.item_start[it] = at; a.p.item_cnt[it] = c; a.p.item_slot[it] = sl; }
            for (int n = 0; n < c; ++n) { s.pair_item[at + n] = it; s.pair_pos[at + n] = n; }
        }
    }
    if (tid == 0) { s.n_items = min(s.tmp[n_vslots], a.p.max_items); s.n_pairs = s.off[n_bins]; }
    __syncthreads();
    // chunks: expert e (bin E = shared expert) owns sorted pairs [off[e], off[e+1]), cut into runs of 8
    for (int e = tid; e < n_bins; e += kFrontThreads) s.tmp[e] = (s.cnt[e] + 7) / 8;
    __syncthreads();
    block_exclusive_scan(s.tmp, n_bins, s.warp_tot);
    for (int e = tid; e < n_bins; e += kFrontThreads) {
        const int first = s.tmp[e], lo = s.off[e], hi = s.off[e + 1];
        for (int q = 0, at = lo; at < hi; ++q, at += 8) {
            const int ch = first + q;
            if (ch < kFrontMaxChunks) { s.chunk_start[ch] = at; s.chunk_cnt[ch] = min(8, hi - at); }
            if (pub && ch < a.p.max_gitems) {
                a.p.gitem_start[ch] = at;
                a.p.gitem_cnt[ch] = min(8, hi - at);
                a.p.gitem_slot[ch] = e < E ? e / K : n_slots;
            }
        }
    }
    if (tid == 0) s.n_chunks = min(min(s.tmp[n_bins], kFrontMaxChunks), a.p.max_gitems);
    __syncthreads();
    if (pub) {
        for (int i = tid; i <= n_bins; i += kFrontThreads) a.p.offsets[i] = s.off[i];
        for (int i = tid; i < s.n_pairs; i += kFrontThreads) {
            a.p.pair_token[i] = s.pair_token[i];
            a.p.pair_expert[i] = s.pair_expert[i];
            a.p.pair_item[i] = s.pair_item[i];
            a.p.pair_pos[i] = s.pair_pos[i];
            a.p.pscale_gu[i] = a.p.tok_scale[s.pair_token[i]];
        }
        if (tid == 0) {
            a.p.counters[0] = s.n_items;
            a.p.counters[1] = s.n_pairs;
            a.p.counters[3] = s.n_chunks;
        }
    }
}

__global__ void __launch_bounds__(kFrontThreads, 1) decode_front_kernel(const FrontArgs a) {
    extern __shared__ __align__(128) uint8_t fsm[];
    __shared__ uint64_t bar;
    __shared__ int hand_off_ok;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // profiling aid: CTA 0 leaves the nanoseconds from its start to the end of each phase in counters[10 ..]
    const uint64_t t_start = globaltimer_ns();
    auto stamp = [&](int idx) {
        if (blockIdx.x == 0 && tid == 0) a.p.counters[10 + idx] = (int32_t)(globaltimer_ns() - t_start);
    };
    if (a.ids_in == nullptr) {
        // ---- phase 0: router logits + token scales, tiles spread over the grid ----
        if (tid == 0) {
            mbar_init(smem_u32(&bar), 1);
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
        __syncthreads();
        const bool ok = a.x_dtype == CHRONOS_DTYPE_BF16 ? front_logits<true>(a, fsm, &bar) : front_logits<false>(a, fsm, &bar);
        stamp(0);
        // every CTA takes part in the hand-off even after a failed copy wait, so that the others do not wait in vain
        const bool all_here = grid_hand_off(a.p.counters + 8, a.p.counters + 2, &hand_off_ok);
        if (!ok || !all_here) return;
        stamp(1);
    }
    FrontPlan& s = *reinterpret_cast<FrontPlan*>(fsm);  // the staging area of phase 0 is free again
    if (a.ids_in == nullptr) {
        // ---- phase 1a: top-k of every token, by every CTA into its own shared memory (identical results everywhere;
        // CTA 0 publishes ids and gates) ----
        TopkArgs tk{a.p.logits, a.L.e_bias, a.L.router_kind, a.L.renorm, a.L.routed_scaling, a.n_tokens, a.L.n_experts,
                    a.L.top_k, s.ids, s.gates};
        for (int t = warp; t < a.n_tokens; t += kFrontWarps) topk_one_token(tk, t, lane);
        __syncthreads();
        if (blockIdx.x == 0)
            for (int i = tid; i < a.n_tokens * a.L.top_k; i += kFrontThreads) { a.p.ids[i] = s.ids[i]; a.p.gates[i] = s.gates[i]; }
        stamp(2);
    } else {
        for (int i = tid; i < a.n_tokens * a.L.top_k; i += kFrontThreads) s.ids[i] = a.ids_in[i];
        __syncthreads();
    }
    // ---- phase 1b: batch coalescing in shared memory ----
    front_plan(a, s);
    stamp(3);
    // ---- phase 2: gate_up input transform of every (pair, 128-column block) into the FP4 activation images ----
    const int H = a.L.hidden;
    {   // the gate_up pass adds the slices of tiles it splits between two CTAs: its output rows start at zero
        float4* z4 = reinterpret_cast<float4*>(a.p.z1);
        const long n4 = (long)s.n_pairs * 2 * a.L.inter / 4;
        for (long i = (long)blockIdx.x * kFrontThreads + tid; i < n4; i += (long)gridDim.x * kFrontThreads) z4[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    // CTA task = a pair: its token's row is staged in shared memory behind the plan (one coalesced read), then warp task =
    // 256-column stage (a 128-block per half-warp, eight values per lane) with the key gathers served from shared memory
    const int nst = H / 256;
    const size_t xb = a.x_dtype == CHRONOS_DTYPE_BF16 ? 2 : 4;
    uint8_t* xrow = fsm + ((sizeof(FrontPlan) + 127) & ~(size_t)127);
    for (int pair = blockIdx.x; pair < s.n_pairs; pair += gridDim.x) {
        const int t = s.pair_token[pair];
        __syncthreads();  // the previous pair's row is no longer read
        {
            const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(a.x) + (size_t)t * H * xb);
            uint4* dst = reinterpret_cast<uint4*>(xrow);
            for (int i = tid; i < (int)(H * xb / 16); i += kFrontThreads) dst[i] = src[i];
        }
        const float gi = 1.0f / a.p.tok_scale[t];
        __syncthreads();
        for (int st = warp; st < nst; st += kFrontWarps) {
            float v[8];
            transform_gu_stage(a.L, xrow, a.x_dtype, 0, s.pair_expert[pair], st, lane, v);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] *= gi;
            uint8_t* img = a.p.bq_gu + ((size_t)s.pair_item[pair] * nst + st) * 6144;
            quantize_stage_fp4x3<32, 8>(v, lane, img, s.pair_pos[pair]);
        }
    }
    __syncthreads();
    stamp(4);
}

// ---------------------------------------------------------------------------------------------------------------
// Between the passes: one CTA per sorted pair.
//   z_gu[i] = beta * r_s1[i] * z1[r_inv[i]] + heal_gu[i];  act = silu(z_gu[:I]) * z_gu[I:]
//   g = power of two near rms(act);  ac = act / g as fp16 (natural order, for the down healer);
//   down-input transform of act / g into the pair's rows of its work item's FP4 image.
// ---------------------------------------------------------------------------------------------------------------
constexpr int kMidThreads = 256;

__global__ void __launch_bounds__(kMidThreads) decode_mid_kernel(const chronos_layer_t L, const Plan p) {
    extern __shared__ __align__(16) float act_s[];  // [I]
    __shared__ float red[kMidThreads / 32];
    __shared__ float g_s;
    const int pair = blockIdx.x;
    // everything that depends on the pair alone is requested at once (the table rows of pairs past the count exist, they
    // just hold old values): the kernel is a chain of memory round trips, and each one taken out of it is ~0.7 us
    const int n_pairs = p.counters[1];
    const int e = p.pair_expert[pair];
    const int item = p.pair_item[pair], pos = p.pair_pos[pair];
    if (pair >= n_pairs) return;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int I = L.inter, E = L.n_experts;
    // the key entries of the down-input transform of this warp's first stage, fetched now and used after the two barriers
    uint4 ce0 = make_uint4(0u, 0u, 0u, 0u);
    uint32_t sw0 = 0u;
    if (e < E && warp < I / 256) {
        const int half = lane >> 4, jl = lane & 15;
        ce0 = *reinterpret_cast<const uint4*>(L.dn_cin + (size_t)e * I + warp * 256 + half * 128 + jl * 8);
        sw0 = L.dn_cs2[(size_t)e * (I / 32) + warp * 8 + half * 4 + (jl >> 2)] >> ((jl & 3) * 8);
    }
    {   // the down pass adds the slices of tiles it splits between two CTAs: this pair's output row starts at zero
        float4* y4 = reinterpret_cast<float4*>(p.y1 + (size_t)pair * L.hidden);
        for (int i = tid; i < L.hidden / 4; i += kMidThreads) y4[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    const float* z1 = p.z1 + (size_t)pair * 2 * I;
    float ss = 0.0f;
    if (e >= E) {  // shared expert: rows in natural order, no healer
        for (int i = tid * 4; i < I; i += kMidThreads * 4) {
            const float4 zg = *reinterpret_cast<const float4*>(z1 + i), zu = *reinterpret_cast<const float4*>(z1 + I + i);
            const float4 av = make_float4(silu_f32(zg.x) * zu.x, silu_f32(zg.y) * zu.y, silu_f32(zg.z) * zu.z, silu_f32(zg.w) * zu.w);
            *reinterpret_cast<float4*>(act_s + i) = av;
            ss += av.x * av.x + av.y * av.y + av.z * av.z + av.w * av.w;
        }
    } else {
        const float beta = L.gu_beta[e];
        const uint16_t* rout = L.gu_rout + (size_t)e * 2 * I;
        const float* heal = p.heal_gu + (size_t)pair * 2 * I;
        for (int i = tid * 4; i < I; i += kMidThreads * 4) {
            const uint2 rg = *reinterpret_cast<const uint2*>(rout + i), ru = *reinterpret_cast<const uint2*>(rout + I + i);
            const float4 hg = *reinterpret_cast<const float4*>(heal + i), hu = *reinterpret_cast<const float4*>(heal + I + i);
            const uint32_t eg[4] = {rg.x & 0xffffu, rg.x >> 16, rg.y & 0xffffu, rg.y >> 16};
            const uint32_t eu[4] = {ru.x & 0xffffu, ru.x >> 16, ru.y & 0xffffu, ru.y >> 16};
            const float hgv[4] = {hg.x, hg.y, hg.z, hg.w}, huv[4] = {hu.x, hu.y, hu.z, hu.w};
            float zgv[4], zuv[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {  // all eight gathers are requested before any is used
                zgv[q] = z1[eg[q] & 0x7fffu];
                zuv[q] = z1[eu[q] & 0x7fffu];
            }
            float av[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float zg = fmaf(beta, (eg[q] >> 15) ? -zgv[q] : zgv[q], hgv[q]);
                const float zu = fmaf(beta, (eu[q] >> 15) ? -zuv[q] : zuv[q], huv[q]);
                av[q] = silu_f32(zg) * zu;
                ss += av[q] * av[q];
            }
            *reinterpret_cast<float4*>(act_s + i) = make_float4(av[0], av[1], av[2], av[3]);
        }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (tid == 0) {
        float tot = 0.0f;
        for (int w = 0; w < kMidThreads / 32; ++w) tot += red[w];  // fixed order
        const float g = pow2_scale(tot, I);
        g_s = g;
        p.pscale_dn[pair] = g;
    }
    __syncthreads();
    const float gi = 1.0f / g_s;
    for (int i = tid * 4; i < I; i += kMidThreads * 4) {
        const float4 a4 = *reinterpret_cast<const float4*>(act_s + i);
        const float s4[4] = {a4.x * gi, a4.y * gi, a4.z * gi, a4.w * gi};
        store_half4(p.ac + (size_t)pair * I + i, s4);
    }
    uint8_t* img0 = p.bq_dn + (size_t)item * (I / 256) * 6144;
    for (int st = warp; st < I / 256; st += kMidThreads / 32) {  // a warp per 256-column stage
        float v[8];
        if (st == warp && e < E) {  // first stage of the warp: its key entries are already here
            const uint32_t ent[8] = {ce0.x & 0xffffu, ce0.x >> 16, ce0.y & 0xffffu, ce0.y >> 16,
                                     ce0.z & 0xffffu, ce0.z >> 16, ce0.w & 0xffffu, ce0.w >> 16};
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float av = act_s[ent[i] & 0x7fffu];
                v[i] = (ent[i] >> 15) ? -av : av;
            }
            fwht128_half(v, lane);
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if ((sw0 >> i) & 1u) v[i] = -v[i];
        } else {
            transform_dn_stage(L, act_s, e, st, lane, v);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] *= gi;
        quantize_stage_fp4x3<32, 8>(v, lane, img0 + (size_t)st * 6144, pos);
    }
}

// ---------------------------------------------------------------------------------------------------------------
// Combine: y[t, i] = sum_j gate[t, j] * (beta_d * r_s1[i] * y1[p_j, r_inv[i]] + heal_dn[p_j, i]) (+ shared expert row),
// j = 0 .. top_k - 1 in that order. One block per (token, 128 output rows), thread = row.
// ---------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(128) decode_combine_kernel(const chronos_layer_t L, const Plan p, const int32_t* __restrict__ ids,
                                                             const float* __restrict__ gates, int with_shared, void* __restrict__ y, int y_dtype) {
    const int t = blockIdx.x, i = blockIdx.y * 128 + threadIdx.x;
    const int H = L.hidden, k = L.top_k;
    float acc = 0.0f;
    for (int j0 = 0; j0 < k; j0 += 8) {
        float term[8], gt[8];
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {  // the loads of up to eight entries are issued together
            const int j = j0 + jj;
            term[jj] = 0.0f;
            gt[jj] = 0.0f;
            if (j >= k) continue;
            const int pos = p.pos_of[t * k + j];
            const int e = ids[t * k + j];  // the entry's expert straight from the routing list: not a second hop after pos
            if (pos < 0) continue;
            const uint32_t ro = L.dn_rout[(size_t)e * H + i];
            const float v = p.y1[(size_t)pos * H + (ro & 0x7fffu)];
            term[jj] = fmaf(L.dn_beta[e], (ro >> 15) ? -v : v, p.heal_dn[(size_t)pos * H + i]);
            gt[jj] = gates[t * k + j];
        }
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) acc = fmaf(gt[jj], term[jj], acc);
    }
    if (with_shared && t >= p.shared_lo && t < p.shared_lo + p.shared_n)
        acc += p.y1[(size_t)(p.offsets[L.n_experts] + t - p.shared_lo) * H + i];
    if (y_dtype == CHRONOS_DTYPE_BF16)
        reinterpret_cast<__nv_bfloat16*>(y)[(size_t)t * H + i] = __float2bfloat16(acc);
    else
        reinterpret_cast<float*>(y)[(size_t)t * H + i] = acc;
}

// ---------------------------------------------------------------------------------------------------------------
static size_t front_smem_bytes(const chronos_layer_t& L, int x_dtype, int tg) {
    const size_t xrow = (size_t)L.hidden * (x_dtype == CHRONOS_DTYPE_BF16 ? 2 : 4);
    const size_t stage = (size_t)kFrontEpc * L.hidden * 4 + (size_t)tg * xrow;
    const size_t plan = ((sizeof(FrontPlan) + 127) & ~(size_t)127) + xrow;  // the plan, then one token row for the input transform
    return stage > plan ? stage : plan;
}

static int front_token_group(const chronos_layer_t& L, int x_dtype, int n_tokens) {
    const size_t budget = 200 * 1024, wrows = (size_t)kFrontEpc * L.hidden * 4, xrow = (size_t)L.hidden * (x_dtype == CHRONOS_DTYPE_BF16 ? 2 : 4);
    if (wrows + xrow > budget) return 0;
    const int fit = (int)((budget - wrows) / xrow);
    return fit < n_tokens ? (fit < 16 ? fit : 16) : (n_tokens < 16 ? n_tokens : 16);
}

// The fused path serves decode-sized batches of the FP4 streaming regime on layers that carry what its kernels read:
// re-tiled banks (p.fp4_stream), healer.v_down as on disk, no tail lattice.
bool decode_fused_fits(const chronos_layer_t& L, int x_dtype, int n_tokens, const Plan& p) {
    return p.fp4_stream && p.heal_gu != nullptr && n_tokens >= 1 && n_tokens <= kFrontMaxTokens && L.tail_bits == 0 &&
           L.v_dn != nullptr && L.n_experts <= 1024 && L.inter <= 8192 && front_token_group(L, x_dtype, n_tokens) >= 1;
}

static size_t g_front_smem_ok[64];  // largest shared-memory footprint the front kernel was found to fit with, per device

int launch_decode_front(const chronos_layer_t& L, const void* x, int x_dtype, int n_tokens, const int32_t* ids_in,
                        int with_shared, const Plan& p, cudaStream_t st) {
    FrontArgs a{};
    a.L = L;
    a.p = p;
    a.x = x;
    a.x_dtype = x_dtype;
    a.n_tokens = n_tokens;
    a.ids_in = ids_in;
    a.with_shared = with_shared;
    a.tg = front_token_group(L, x_dtype, n_tokens);
    const size_t smem = front_smem_bytes(L, x_dtype, a.tg);
    if (int rc = ensure_dynamic_smem(reinterpret_cast<const void*>(decode_front_kernel), smem, "decode_front")) return rc;
    int dev = 0;
    cudaGetDevice(&dev);
    const int grid = device_sm_count();  // one CTA per SM
    if (dev < 0 || dev >= 64 || g_front_smem_ok[dev] < smem) {
        // the grid-wide hand-off needs every CTA resident at once: check that an SM holds a CTA of this footprint
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_front_kernel, kFrontThreads, smem) != cudaSuccess || per_sm < 1) {
            cudaGetLastError();
            set_error("decode_front: an SM cannot hold a CTA of %d threads with %zu bytes of shared memory", kFrontThreads, smem);
            return CHRONOS_E_LAUNCH;
        }
        if (dev >= 0 && dev < 64) g_front_smem_ok[dev] = smem;
    }
    void* params[] = {(void*)&a};
    const cudaError_t rc = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(decode_front_kernel), dim3((unsigned)grid), dim3(kFrontThreads),
                                                       params, smem, st);
    if (rc != cudaSuccess) {
        cudaGetLastError();
        set_error("decode_front: cooperative launch refused: %s", cudaGetErrorString(rc));
        return CHRONOS_E_LAUNCH;
    }
    return check_launch("decode_front");
}

int launch_decode_mid(const chronos_layer_t& L, const Plan& p, cudaStream_t st) {
    decode_mid_kernel<<<(unsigned)p.max_pairs, kMidThreads, (size_t)L.inter * 4, st>>>(L, p);
    return check_launch("decode_mid");
}

int launch_decode_combine(const chronos_layer_t& L, const Plan& p, const int32_t* ids, const float* gates, int n_tokens, int with_shared,
                          void* y, int y_dtype, cudaStream_t st) {
    if (n_tokens <= 0) return CHRONOS_OK;
    decode_combine_kernel<<<dim3((unsigned)n_tokens, (unsigned)(L.hidden / 128)), 128, 0, st>>>(L, p, ids, gates, with_shared && L.shared_inter > 0, y,
                                                                                                y_dtype);
    return check_launch("decode_combine");
}

}  // namespace chronos
