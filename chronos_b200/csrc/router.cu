// Router: fp32 logits in a fixed, reproducible summation order + top-k + gate weights.
#include <algorithm>

#include "common.cuh"

namespace chronos {

// logits[t, e] = sum_k x[t, k] * w[e, k] in ONE stated order, so that the CPU oracle can reproduce every bit:
// lane l (0..31) accumulates, by fused multiply-add starting from +0, the products at k = 128 j + 4 l + i for
// j = 0, 1, ... and i = 0..3 (j ascending, then i); the 32 lane sums are combined by the xor butterfly 16, 8, 4, 2, 1.
// Any tiling gives the same bits because every (t, e) dot is owned by one warp and walks k in that order; the order
// lets a lane fetch its four consecutive columns with one vector load. Each warp computes a TOK-token x EXP-expert
// tile: (4, 1) spreads decode-sized batches over many warps, (4, 4) reuses loaded operands for prefill-sized ones.
template <bool BF16>
__device__ __forceinline__ float4 ld_x4(const void* x, size_t i) {
    if (BF16) {
        const uint2 v = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(x) + i);
        return make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u), __uint_as_float(v.y << 16),
                           __uint_as_float(v.y & 0xffff0000u));
    }
    return *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + i);
}

template <int TOK, int EXP, bool BF16>
__global__ void __launch_bounds__(256) router_logits_kernel(const void* __restrict__ x, const float* __restrict__ w,
                                                            float* __restrict__ logits, int n_tokens, int n_experts,
                                                            int hidden, float* __restrict__ tok_scale) {
    const int lane = threadIdx.x & 31;
    const int warp_in_block = threadIdx.x >> 5;
    const int e_tiles = (n_experts + EXP - 1) / EXP;
    const int t_tiles = (n_tokens + TOK - 1) / TOK;
    const long tile = (long)blockIdx.x * 8 + warp_in_block;
    if (tile >= (long)e_tiles * t_tiles) return;
    // consecutive warps of a block share the token tile (x stays in L1) and walk over expert tiles
    const int tt = (int)(tile / e_tiles), et = (int)(tile % e_tiles);
    const int t0 = tt * TOK, e0 = et * EXP;
    float acc[TOK][EXP];
    float ssq[TOK];
#pragma unroll
    for (int a = 0; a < TOK; ++a) {
        ssq[a] = 0.0f;
#pragma unroll
        for (int b = 0; b < EXP; ++b) acc[a][b] = 0.0f;
    }
    size_t xoff[TOK], woff[EXP];
#pragma unroll
    for (int a = 0; a < TOK; ++a) xoff[a] = (size_t)min(t0 + a, n_tokens - 1) * hidden + 4 * lane;
#pragma unroll
    for (int b = 0; b < EXP; ++b) woff[b] = (size_t)min(e0 + b, n_experts - 1) * hidden + 4 * lane;
    // the warp that owns expert tile 0 of a token tile also produces the tokens' power-of-two activation scales
    // (near rms(x[t])): it reads every x element anyway
    const bool do_scale = tok_scale != nullptr && et == 0;
    // 128-column steps whose loads are issued together (the FMA order per dot is unchanged); the 8 x 8 tile already holds 64
    // accumulators and 16 vector loads per step
    constexpr int UN = EXP == 1 ? 8 : (TOK * EXP > 16 ? 1 : 4);
    int k = 0;
    for (; k + UN * 128 <= hidden; k += UN * 128) {
        float4 xv[UN][TOK], wv[UN][EXP];
#pragma unroll
        for (int u = 0; u < UN; ++u) {
#pragma unroll
            for (int a = 0; a < TOK; ++a) xv[u][a] = ld_x4<BF16>(x, xoff[a] + k + u * 128);
#pragma unroll
            for (int b = 0; b < EXP; ++b) wv[u][b] = *reinterpret_cast<const float4*>(w + woff[b] + k + u * 128);
        }
#pragma unroll
        for (int u = 0; u < UN; ++u)
#pragma unroll
            for (int a = 0; a < TOK; ++a) {
#pragma unroll
                for (int b = 0; b < EXP; ++b) {
                    acc[a][b] = __fmaf_rn(xv[u][a].x, wv[u][b].x, acc[a][b]);
                    acc[a][b] = __fmaf_rn(xv[u][a].y, wv[u][b].y, acc[a][b]);
                    acc[a][b] = __fmaf_rn(xv[u][a].z, wv[u][b].z, acc[a][b]);
                    acc[a][b] = __fmaf_rn(xv[u][a].w, wv[u][b].w, acc[a][b]);
                }
                ssq[a] = fmaf(xv[u][a].x, xv[u][a].x, fmaf(xv[u][a].y, xv[u][a].y, fmaf(xv[u][a].z, xv[u][a].z, fmaf(xv[u][a].w, xv[u][a].w, ssq[a]))));
            }
    }
    for (; k < hidden; k += 128) {
#pragma unroll
        for (int a = 0; a < TOK; ++a) {
            const float4 xq = ld_x4<BF16>(x, xoff[a] + k);
#pragma unroll
            for (int b = 0; b < EXP; ++b) {
                const float4 wq = *reinterpret_cast<const float4*>(w + woff[b] + k);
                acc[a][b] = __fmaf_rn(xq.x, wq.x, acc[a][b]);
                acc[a][b] = __fmaf_rn(xq.y, wq.y, acc[a][b]);
                acc[a][b] = __fmaf_rn(xq.z, wq.z, acc[a][b]);
                acc[a][b] = __fmaf_rn(xq.w, wq.w, acc[a][b]);
            }
            ssq[a] = fmaf(xq.x, xq.x, fmaf(xq.y, xq.y, fmaf(xq.z, xq.z, fmaf(xq.w, xq.w, ssq[a]))));
        }
    }
    if (do_scale) {
#pragma unroll
        for (int a = 0; a < TOK; ++a) {
            float v = ssq[a];
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            if (lane == 0 && t0 + a < n_tokens) {
                const float rms = sqrtf(v / (float)hidden);
                tok_scale[t0 + a] = rms > 0.0f ? exp2f(rintf(log2f(rms))) : 1.0f;
            }
        }
    }
#pragma unroll
    for (int a = 0; a < TOK; ++a)
#pragma unroll
        for (int b = 0; b < EXP; ++b) {
            float v = acc[a][b];
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
            if (lane == 0 && t0 + a < n_tokens && e0 + b < n_experts) logits[(size_t)(t0 + a) * n_experts + e0 + b] = v;
        }
}

// Large batches: the same dots from shared memory. A CTA of 16 warps computes 64 tokens x 16 experts; per 128-column
// step it stages the 64 activation rows (in their own dtype) and the 16 router rows with 16-byte asynchronous copies
// into an 8-deep ring, and warp (wt, we) multiplies tokens 8 wt .. + 7 by experts 8 we .. + 7 in the stated order
// (lane l: k = 128 j + 4 l + i). Global traffic per logit drops from 3 KB (register tile straight from L2) to 24 B
// per step, which is what bounded the register-tile kernel on large batches. Bits are identical to the other kernels.
constexpr int kRtTok = 64, kRtExp = 16, kRtThreads = 512;
constexpr int kRtStagesBf16 = 8, kRtStagesF32 = 5;  // steps in flight: enough to cover the L2 latency, bounded by shared memory

template <bool BF16, bool SCALE>  // SCALE: the CTAs of the first expert tile also produce the token scales
__global__ void __launch_bounds__(kRtThreads) router_logits_tiled_kernel(const void* __restrict__ x, const float* __restrict__ w,
                                                                         float* __restrict__ logits, int n_tokens, int n_experts,
                                                                         int hidden, float* __restrict__ tok_scale) {
    extern __shared__ __align__(16) uint8_t rts[];
    constexpr int XB = BF16 ? 2 : 4;
    constexpr int kRtStages = BF16 ? kRtStagesBf16 : kRtStagesF32;
    constexpr int XS = kRtTok * 128 * XB, WS = kRtExp * 128 * 4, STAGE = XS + WS;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int wt = warp >> 1, we = warp & 1;
    const int e_tiles = (n_experts + kRtExp - 1) / kRtExp;
    const int t0 = (int)(blockIdx.x / e_tiles) * kRtTok, e0 = (int)(blockIdx.x % e_tiles) * kRtExp;
    const int n_steps = hidden / 128;
    auto stage_in = [&](int step) {
        uint8_t* dst = rts + (size_t)(step % kRtStages) * STAGE;
        // activations: 64 rows x (128 * XB / 16) chunks; router rows: 16 rows x 32 chunks
        constexpr int XC = 128 * XB / 16;
        for (int c = tid; c < kRtTok * XC; c += kRtThreads) {
            const int row = c / XC, ch = c % XC;
            const int t = min(t0 + row, n_tokens - 1);
            const uint8_t* src = reinterpret_cast<const uint8_t*>(x) + ((size_t)t * hidden + (size_t)step * 128) * XB + ch * 16;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst + row * 128 * XB + ch * 16)), "l"(src) : "memory");
        }
        for (int c = tid; c < kRtExp * 32; c += kRtThreads) {
            const int row = c / 32, ch = c % 32;
            const int e = min(e0 + row, n_experts - 1);
            const float* src = w + (size_t)e * hidden + (size_t)step * 128 + ch * 4;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst + XS + row * 512 + ch * 16)), "l"(src) : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    float acc[8][8], ssq[8];
#pragma unroll
    for (int a = 0; a < 8; ++a) {
        ssq[a] = 0.0f;
#pragma unroll
        for (int b = 0; b < 8; ++b) acc[a][b] = 0.0f;
    }
    const bool do_scale = SCALE && tok_scale != nullptr && e0 == 0 && we == 0;
    for (int s = 0; s < kRtStages - 1; ++s) {
        if (s < n_steps) stage_in(s);
        else asm volatile("cp.async.commit_group;" ::: "memory");
    }
    for (int step = 0; step < n_steps; ++step) {
        asm volatile("cp.async.wait_group %0;" ::"n"(kRtStages - 2) : "memory");
        __syncthreads();  // the step's bytes have landed for every thread; the slot refilled below was read a step ago
        if (step + kRtStages - 1 < n_steps) stage_in(step + kRtStages - 1);
        else asm volatile("cp.async.commit_group;" ::: "memory");
        const uint8_t* cur = rts + (size_t)(step % kRtStages) * STAGE;
        float4 wv[8];
#pragma unroll
        for (int b = 0; b < 8; ++b) wv[b] = *reinterpret_cast<const float4*>(cur + XS + (we * 8 + b) * 512 + lane * 16);
#pragma unroll
        for (int a = 0; a < 8; ++a) {
            float4 xq;
            if (BF16) {
                const uint2 u = *reinterpret_cast<const uint2*>(cur + (wt * 8 + a) * 256 + lane * 8);
                xq = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                                 __uint_as_float(u.y & 0xffff0000u));
            } else {
                xq = *reinterpret_cast<const float4*>(cur + (wt * 8 + a) * 512 + lane * 16);
            }
#pragma unroll
            for (int b = 0; b < 8; ++b) {
                acc[a][b] = __fmaf_rn(xq.x, wv[b].x, acc[a][b]);
                acc[a][b] = __fmaf_rn(xq.y, wv[b].y, acc[a][b]);
                acc[a][b] = __fmaf_rn(xq.z, wv[b].z, acc[a][b]);
                acc[a][b] = __fmaf_rn(xq.w, wv[b].w, acc[a][b]);
            }
            if (SCALE && do_scale) ssq[a] = fmaf(xq.x, xq.x, fmaf(xq.y, xq.y, fmaf(xq.z, xq.z, fmaf(xq.w, xq.w, ssq[a]))));  // warp-uniform
        }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    const int tw = t0 + wt * 8, ew = e0 + we * 8;
    if (do_scale) {
#pragma unroll
        for (int a = 0; a < 8; ++a) {
            float v = ssq[a];
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            if (lane == 0 && tw + a < n_tokens) {
                const float rms = sqrtf(v / (float)hidden);
                tok_scale[tw + a] = rms > 0.0f ? exp2f(rintf(log2f(rms))) : 1.0f;
            }
        }
    }
#pragma unroll
    for (int a = 0; a < 8; ++a)
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            float v = acc[a][b];
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
            if (lane == 0 && tw + a < n_tokens && ew + b < n_experts) logits[(size_t)(tw + a) * n_experts + ew + b] = v;
        }
}

// Decode-sized batches: the dots are few and every one is a long dependent walk over k, so the time is pure memory
// latency. One CTA stages EPC router rows and up to 4 activation rows in shared memory with bulk async copies
// (all bytes requested at once, one wait), then warp w computes expert e0 + w against the 4 tokens in the stated
// order (lane l: k = 128 j + 4 l + i). Bits are identical to router_logits_kernel.
template <bool BF16>
__global__ void __launch_bounds__(256) router_logits_small_kernel(const void* __restrict__ x, const float* __restrict__ w,
                                                                  float* __restrict__ logits, int n_tokens, int n_experts,
                                                                  int hidden, int epc, float* __restrict__ tok_scale,
                                                                  int32_t* __restrict__ status) {
    extern __shared__ __align__(128) uint8_t rsm[];
    __shared__ uint64_t bar;
    constexpr int XB = BF16 ? 2 : 4;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int e_tiles = (n_experts + epc - 1) / epc;
    const int tt = blockIdx.x / e_tiles, et = blockIdx.x % e_tiles;
    const int t0 = tt * 4, e0 = et * epc;
    const int nt = min(4, n_tokens - t0), ne = min(epc, n_experts - e0);
    float* ws = reinterpret_cast<float*>(rsm);                       // [epc][hidden]
    uint8_t* xs = rsm + (size_t)epc * hidden * 4;                    // [4][hidden] in the activation dtype
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bar), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        mbar_expect_tx(smem_u32(&bar), (uint32_t)(ne * hidden * 4 + nt * hidden * XB));
        for (int i = 0; i < ne; ++i)
            bulk_g2s(smem_u32(ws + (size_t)i * hidden), w + (size_t)(e0 + i) * hidden, (uint32_t)hidden * 4, smem_u32(&bar));
        for (int a = 0; a < nt; ++a)
            bulk_g2s(smem_u32(xs + (size_t)a * hidden * XB), reinterpret_cast<const uint8_t*>(x) + (size_t)(t0 + a) * hidden * XB,
                     (uint32_t)hidden * XB, smem_u32(&bar));
    }
    __syncthreads();
    const bool ok = mbar_wait(smem_u32(&bar), 0);
    if (__syncthreads_or(!ok)) {
        if (threadIdx.x == 0) atomicOr(status, kStatusRouterTimeout);
        return;
    }
    for (int ew = warp; ew < ne; ew += 8) {
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f}, ssq[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const float* wr = ws + (size_t)ew * hidden + 4 * lane;
        for (int k = 0; k < hidden; k += 128) {
            const float4 wq = *reinterpret_cast<const float4*>(wr + k);
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                if (a < nt) {
                    float4 xq;
                    if (BF16) {
                        const uint2 v = *reinterpret_cast<const uint2*>(xs + ((size_t)a * hidden + k + 4 * lane) * 2);
                        xq = make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u),
                                         __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xffff0000u));
                    } else {
                        xq = *reinterpret_cast<const float4*>(xs + ((size_t)a * hidden + k + 4 * lane) * 4);
                    }
                    acc[a] = __fmaf_rn(xq.x, wq.x, acc[a]);
                    acc[a] = __fmaf_rn(xq.y, wq.y, acc[a]);
                    acc[a] = __fmaf_rn(xq.z, wq.z, acc[a]);
                    acc[a] = __fmaf_rn(xq.w, wq.w, acc[a]);
                    ssq[a] = fmaf(xq.x, xq.x, fmaf(xq.y, xq.y, fmaf(xq.z, xq.z, fmaf(xq.w, xq.w, ssq[a]))));
                }
            }
        }
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            float v = acc[a];
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
            if (lane == 0 && a < nt) logits[(size_t)(t0 + a) * n_experts + e0 + ew] = v;
            if (tok_scale != nullptr && et == 0 && ew == 0) {
                float q = ssq[a];
#pragma unroll
                for (int off = 16; off >= 1; off >>= 1) q += __shfl_xor_sync(0xffffffffu, q, off);
                if (lane == 0 && a < nt) {
                    const float rms = sqrtf(q / (float)hidden);
                    tok_scale[t0 + a] = rms > 0.0f ? exp2f(rintf(log2f(rms))) : 1.0f;
                }
            }
        }
    }
}

// One warp per token: k rounds of arg-max over the choice scores (ties -> lower index), then the gate weights.
// softmax flavour: choice = logit, gate = softmax over the k chosen logits.
// sigmoid flavour: choice = sigmoid(logit) + bias, weight = sigmoid(logit) (unbiased), optional renorm, * scaling.
// (topk_one_token lives in common.cuh so that the plan kernel can run it in the same launch.)
__global__ void __launch_bounds__(256) router_topk_kernel(TopkArgs tk) {
    const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (t >= tk.n_tokens) return;
    topk_one_token(tk, t, threadIdx.x & 31);
}

// ---------------------------------------------------------------------------------------------------------------
// Batch-coalesced routing policy for speculative verify batches (streams of `tps` tokens: one anchor + drafts).
// Only a prose description of the policy exists in the reference (README.md:56, :208, :372 and
// docs/CHRONOS_ARCHITECTURE_PAPER.md:270-277; its kernel lives in another repository), so this is a clean-room design
// that keeps the stated invariants:
//   * the anchor (token 0 of a stream) gets its natural top-k, untouched;
//   * a draft token only ever picks from its own natural top-`pool` candidates (pool >= k);
//   * its `keep` best natural experts are always kept, in natural order;
//   * the remaining k - keep picks go to the candidates ranked by (choice score + bonus if the anchor selected the
//     expert too), ties to the better natural rank - so experts whose bank the anchor already streams are preferred;
//   * pool == k (or bonus == 0) gives natural routing; gate weights come from the unbiased scores of what was picked.
// One CTA per stream: warp 0 routes the anchor, then one warp per draft.
// ---------------------------------------------------------------------------------------------------------------
template <int PL>
__device__ __forceinline__ void natural_ranking(const TopkArgs& a, int t, int lane, int n_rounds, int& my_id, float& my_choice) {
    float choice[PL];
#pragma unroll
    for (int i = 0; i < PL; ++i) {
        const int e = i * 32 + lane;
        float c = -INFINITY;
        if (e < a.n_experts) {
            c = router_choice(a, a.logits[(size_t)t * a.n_experts + e], e);
            if (!(c == c)) c = -INFINITY;
        }
        choice[i] = c;
    }
    my_id = -1;
    my_choice = -INFINITY;
    for (int j = 0; j < n_rounds; ++j) {  // lane j keeps the j-th best candidate
        float best;
        int best_e;
        lane_argmax<PL>(choice, lane, best, best_e);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, off);
            const int oe = __shfl_xor_sync(0xffffffffu, best_e, off);
            if (ov > best || (ov == best && oe < best_e)) { best = ov; best_e = oe; }
        }
        const bool found = best_e != kNoExpert;
#pragma unroll
        for (int i = 0; i < PL; ++i)
            if (found && i * 32 + lane == best_e) choice[i] = -INFINITY;
        if (lane == j && found) { my_id = best_e; my_choice = best; }
    }
}

__device__ __forceinline__ void write_gates(const TopkArgs& a, int t, int lane, int my_id) {
    // lane j < top_k holds the j-th selected expert (or -1); gate weights per flavour from the unbiased scores
    const bool have = lane < a.top_k && my_id >= 0;
    float my_val = 0.0f;
    if (have) my_val = router_weight_source(a, a.logits[(size_t)t * a.n_experts + my_id]);
    float gate;
    if (a.kind != CHRONOS_ROUTER_SOFTMAX_TOPK) {
        const float sv = have ? my_val : 0.0f;
        float tot = 0.0f;
        for (int j = 0; j < a.top_k; ++j) tot += __shfl_sync(0xffffffffu, sv, j);
        gate = (a.renorm ? my_val / (tot + 1e-20f) : my_val) * a.scaling;
    } else {
        float mx = have ? my_val : -INFINITY;  // the picks of a draft are not sorted by logit: take the maximum explicitly
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
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

template <int PL>
__global__ void __launch_bounds__(256) coalesced_topk_kernel(TopkArgs a, int tps, int pool, int keep, float bonus) {
    __shared__ int anchor_ids[kMaxTopK];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, n_warps = blockDim.x >> 5;
    const int t0 = blockIdx.x * tps;
    if (warp == 0) {
        int id;
        float c;
        natural_ranking<PL>(a, t0, lane, a.top_k, id, c);
        if (lane < a.top_k) anchor_ids[lane] = id;
        write_gates(a, t0, lane, id);
    }
    __syncthreads();
    for (int m = 1 + warp; m < tps; m += n_warps) {
        const int t = t0 + m;
        if (t >= a.n_tokens) break;
        int id;
        float c;
        natural_ranking<PL>(a, t, lane, pool, id, c);  // lane j: j-th natural candidate
        bool shared_with_anchor = false;
        for (int j = 0; j < a.top_k; ++j) shared_with_anchor |= (id >= 0 && anchor_ids[j] == id);
        const bool cand = lane >= keep && lane < pool && id >= 0;
        const float sc = cand ? c + (shared_with_anchor ? bonus : 0.0f) : -INFINITY;
        int rank = 0;  // candidates that come before this lane's
        for (int j = 0; j < 32; ++j) {
            const float oj = __shfl_sync(0xffffffffu, sc, j);
            rank += (oj > sc) || (oj == sc && j < lane);
        }
        // output position: kept candidates stay where they are, the others go by rank behind them
        const int out_pos = lane < keep ? lane : (cand ? keep + rank : 32);
        int sel_id = -1;
        for (int j = 0; j < 32; ++j) {  // lane p takes the id of the lane whose output position is p
            const int pj = __shfl_sync(0xffffffffu, out_pos, j);
            const int ij = __shfl_sync(0xffffffffu, id, j);
            if (pj == lane) sel_id = ij;
        }
        write_gates(a, t, lane, lane < a.top_k ? sel_id : -1);
    }
}

int launch_coalesced_topk(const chronos_layer_t& L, const float* logits, int n_tokens, int tps, int pool, int keep, float bonus,
                          int32_t* ids, float* gates, cudaStream_t st) {
    TopkArgs tk{logits, L.e_bias, L.router_kind, L.renorm, L.routed_scaling, n_tokens, L.n_experts, L.top_k, ids, gates};
    const unsigned grid = (unsigned)((n_tokens + tps - 1) / tps);
    const int threads = 32 * (tps < 8 ? tps : 8);
    if (L.n_experts <= 256) coalesced_topk_kernel<8><<<grid, threads, 0, st>>>(tk, tps, pool, keep, bonus);
    else if (L.n_experts <= 320) coalesced_topk_kernel<10><<<grid, threads, 0, st>>>(tk, tps, pool, keep, bonus);
    else if (L.n_experts <= 512) coalesced_topk_kernel<16><<<grid, threads, 0, st>>>(tk, tps, pool, keep, bonus);
    else coalesced_topk_kernel<32><<<grid, threads, 0, st>>>(tk, tps, pool, keep, bonus);
    return check_launch("coalesced_topk");
}

int launch_router(const chronos_layer_t& L, const void* x, int x_dtype, int n_tokens, int32_t* ids, float* gates,
                  float* logits, float* tok_scale, int32_t* status, cudaStream_t st) {
    if (n_tokens <= 0) return CHRONOS_OK;
    const bool bf16 = x_dtype == CHRONOS_DTYPE_BF16;
    const size_t xrow = (size_t)L.hidden * (bf16 ? 2 : 4), wrow = (size_t)L.hidden * 4;
    // router rows per CTA of the shared-memory kernel: what is left of 200 KiB after 4 activation rows; 0 (rows too
    // long to stage, e.g. hidden 16384 in fp32) selects the register-tile kernel below
    const size_t stage_budget = 200 * 1024;
    const int epc = 4 * xrow + wrow <= stage_budget ? (int)std::min<size_t>(8, (stage_budget - 4 * xrow) / wrow) : 0;
    if (n_tokens <= 64 && epc >= 1 && status != nullptr) {
        const size_t smem = (size_t)epc * wrow + 4 * xrow;
        const unsigned grid = (unsigned)(((L.n_experts + epc - 1) / epc) * ((n_tokens + 3) / 4));
        if (int rc = ensure_dynamic_smem(bf16 ? reinterpret_cast<const void*>(router_logits_small_kernel<true>)
                                              : reinterpret_cast<const void*>(router_logits_small_kernel<false>), smem, "router")) return rc;
        if (bf16) router_logits_small_kernel<true><<<grid, 256, smem, st>>>(x, L.router_w, logits, n_tokens, L.n_experts, L.hidden, epc, tok_scale, status);
        else router_logits_small_kernel<false><<<grid, 256, smem, st>>>(x, L.router_w, logits, n_tokens, L.n_experts, L.hidden, epc, tok_scale, status);
    } else if (n_tokens <= 64) {
        const long tiles = (long)L.n_experts * ((n_tokens + 3) / 4);
        const unsigned grid = (unsigned)((tiles + 7) / 8);
        if (bf16) router_logits_kernel<4, 1, true><<<grid, 256, 0, st>>>(x, L.router_w, logits, n_tokens, L.n_experts, L.hidden, tok_scale);
        else router_logits_kernel<4, 1, false><<<grid, 256, 0, st>>>(x, L.router_w, logits, n_tokens, L.n_experts, L.hidden, tok_scale);
    } else if (n_tokens >= 256) {  // large batches: shared-memory tiles of 64 tokens x 16 experts
        const unsigned grid = (unsigned)(((n_tokens + kRtTok - 1) / kRtTok) * ((L.n_experts + kRtExp - 1) / kRtExp));
        const size_t smem = (size_t)(bf16 ? kRtStagesBf16 : kRtStagesF32) * (kRtTok * 128 * (bf16 ? 2 : 4) + kRtExp * 512);
        // the token scales come from a kernel of their own here: carrying eight more sums per lane through the tile loop
        // spilled registers in every CTA for the sake of one expert tile in eighteen
        if (int rc = ensure_dynamic_smem(bf16 ? reinterpret_cast<const void*>(router_logits_tiled_kernel<true, false>)
                                              : reinterpret_cast<const void*>(router_logits_tiled_kernel<false, false>), smem, "router")) return rc;
        if (bf16) router_logits_tiled_kernel<true, false><<<grid, kRtThreads, smem, st>>>(x, L.router_w, logits, n_tokens, L.n_experts, L.hidden, nullptr);
        else router_logits_tiled_kernel<false, false><<<grid, kRtThreads, smem, st>>>(x, L.router_w, logits, n_tokens, L.n_experts, L.hidden, nullptr);
        if (tok_scale != nullptr)
            if (int rc = launch_token_scale(x, x_dtype, n_tokens, L.hidden, tok_scale, st)) return rc;
    } else {
        const long tiles = (long)((L.n_experts + 3) / 4) * ((n_tokens + 3) / 4);
        const unsigned grid = (unsigned)((tiles + 7) / 8);
        if (bf16) router_logits_kernel<4, 4, true><<<grid, 256, 0, st>>>(x, L.router_w, logits, n_tokens, L.n_experts, L.hidden, tok_scale);
        else router_logits_kernel<4, 4, false><<<grid, 256, 0, st>>>(x, L.router_w, logits, n_tokens, L.n_experts, L.hidden, tok_scale);
    }
    if (int rc = check_launch("router_logits")) return rc;
    if (ids == nullptr) return CHRONOS_OK;  // the caller runs the top-k inside its plan launch
    TopkArgs tk{logits, L.e_bias, L.router_kind, L.renorm, L.routed_scaling, n_tokens, L.n_experts, L.top_k, ids, gates};
    router_topk_kernel<<<(unsigned)((n_tokens + 7) / 8), 256, 0, st>>>(tk);
    return check_launch("router_topk");
}

}  // namespace chronos
