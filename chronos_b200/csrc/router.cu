// Router: fp32 logits in a fixed, reproducible summation order + top-k + gate weights.
#include "common.cuh"

namespace chronos {

// logits[t, e] = sum_k x[t, k] * w[e, k] with lane l accumulating k = l, l+32, ... ascending by FMA from +0,
// lanes combined by the xor butterfly 16, 8, 4, 2, 1. Any tiling gives the same bits because every (t, e) dot is
// owned by one warp and walks k in that order. Each warp computes a TOK-token x EXP-expert tile: (4, 1) spreads
// decode-sized batches over many warps, (4, 4) reuses loaded operands for prefill-sized ones.
template <int TOK, int EXP>
__global__ void __launch_bounds__(256) router_logits_kernel(const void* __restrict__ x, int x_dtype,
                                                            const float* __restrict__ w, float* __restrict__ logits,
                                                            int n_tokens, int n_experts, int hidden,
                                                            float* __restrict__ tok_scale) {
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
#pragma unroll
    for (int a = 0; a < TOK; ++a)
#pragma unroll
        for (int b = 0; b < EXP; ++b) acc[a][b] = 0.0f;
    size_t xoff[TOK], woff[EXP];
#pragma unroll
    for (int a = 0; a < TOK; ++a) xoff[a] = (size_t)min(t0 + a, n_tokens - 1) * hidden;
#pragma unroll
    for (int b = 0; b < EXP; ++b) woff[b] = (size_t)min(e0 + b, n_experts - 1) * hidden;
    // the warp that owns expert tile 0 of a token tile also produces the tokens' power-of-two activation scales
    // (near rms(x[t])): it reads every x element anyway
    const bool do_scale = tok_scale != nullptr && et == 0;
    float ssq[TOK];
#pragma unroll
    for (int a = 0; a < TOK; ++a) ssq[a] = 0.0f;
    constexpr int UN = 8;  // k-steps whose loads are issued together (the FMA order per dot is unchanged)
    int k = lane;
    for (; k + (UN - 1) * 32 < hidden; k += UN * 32) {
        float xv[UN][TOK], wv[UN][EXP];
#pragma unroll
        for (int u = 0; u < UN; ++u) {
#pragma unroll
            for (int a = 0; a < TOK; ++a) xv[u][a] = ld_act(x, x_dtype, xoff[a] + k + u * 32);
#pragma unroll
            for (int b = 0; b < EXP; ++b) wv[u][b] = w[woff[b] + k + u * 32];
        }
#pragma unroll
        for (int u = 0; u < UN; ++u)
#pragma unroll
            for (int a = 0; a < TOK; ++a) {
#pragma unroll
                for (int b = 0; b < EXP; ++b) acc[a][b] = __fmaf_rn(xv[u][a], wv[u][b], acc[a][b]);
                ssq[a] = fmaf(xv[u][a], xv[u][a], ssq[a]);
            }
    }
    for (; k < hidden; k += 32) {
#pragma unroll
        for (int a = 0; a < TOK; ++a) {
            const float xv1 = ld_act(x, x_dtype, xoff[a] + k);
#pragma unroll
            for (int b = 0; b < EXP; ++b) acc[a][b] = __fmaf_rn(xv1, w[woff[b] + k], acc[a][b]);
            ssq[a] = fmaf(xv1, xv1, ssq[a]);
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

// One warp per token: k rounds of arg-max over the choice scores (ties -> lower index), then the gate weights.
// softmax flavour: choice = logit, gate = softmax over the k chosen logits.
// sigmoid flavour: choice = sigmoid(logit) + bias, weight = sigmoid(logit) (unbiased), optional renorm, * scaling.
__global__ void __launch_bounds__(256) router_topk_kernel(const float* __restrict__ logits,
                                                          const float* __restrict__ e_bias, int kind, int renorm,
                                                          float scaling, int n_tokens, int n_experts, int top_k,
                                                          int32_t* __restrict__ ids, float* __restrict__ gates) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (t >= n_tokens) return;
    constexpr int kMaxPerLane = 32;  // n_experts <= 1024
    float choice[kMaxPerLane];
    const int per_lane = (n_experts + 31) / 32;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
        const int e = i * 32 + lane;
        float c = -INFINITY;
        if (i < per_lane && e < n_experts) {
            const float lg = logits[(size_t)t * n_experts + e];
            c = kind == CHRONOS_ROUTER_SIGMOID_NOAUX ? (1.0f / (1.0f + expf(-lg))) + (e_bias ? e_bias[e] : 0.0f) : lg;
        }
        choice[i] = c;
    }
    float my_val = 0.0f;  // lane j keeps the j-th chosen weight source
    int my_id = -1;
    for (int j = 0; j < top_k; ++j) {
        float best = -INFINITY;
        int best_e = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) {
            const int e = i * 32 + lane;
            if (i < per_lane && e < n_experts && (choice[i] > best)) { best = choice[i]; best_e = e; }
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, off);
            const int oe = __shfl_xor_sync(0xffffffffu, best_e, off);
            if (ov > best || (ov == best && oe < best_e)) { best = ov; best_e = oe; }
        }
        // remove the winner from its owner lane
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i)
            if (i * 32 + lane == best_e) choice[i] = -INFINITY;
        if (lane == j) {
            my_id = best_e;
            const float lg = logits[(size_t)t * n_experts + best_e];
            my_val = kind == CHRONOS_ROUTER_SIGMOID_NOAUX ? 1.0f / (1.0f + expf(-lg)) : lg;
        }
    }
    float gate;
    if (kind == CHRONOS_ROUTER_SIGMOID_NOAUX) {
        float s = lane < top_k ? my_val : 0.0f;
        // sequential sum in index order, the way a row reduction over k values reads
        float tot = 0.0f;
        for (int j = 0; j < top_k; ++j) tot += __shfl_sync(0xffffffffu, s, j);
        gate = renorm ? my_val / (tot + 1e-20f) : my_val;
        gate *= scaling;
    } else {
        const float mx = __shfl_sync(0xffffffffu, my_val, 0);  // chosen values are in descending order
        const float ex = lane < top_k ? expf(my_val - mx) : 0.0f;
        float tot = 0.0f;
        for (int j = 0; j < top_k; ++j) tot += __shfl_sync(0xffffffffu, ex, j);
        gate = ex / tot;
    }
    if (lane < top_k) {
        ids[(size_t)t * top_k + lane] = my_id;
        gates[(size_t)t * top_k + lane] = gate;
    }
}

int launch_router(const chronos_layer_t& L, const void* x, int x_dtype, int n_tokens, int32_t* ids, float* gates,
                  float* logits, float* tok_scale, cudaStream_t st) {
    if (n_tokens <= 0) return CHRONOS_OK;
    if (n_tokens <= 64) {
        const long tiles = (long)L.n_experts * ((n_tokens + 3) / 4);
        router_logits_kernel<4, 1><<<(unsigned)((tiles + 7) / 8), 256, 0, st>>>(x, x_dtype, L.router_w, logits, n_tokens,
                                                                               L.n_experts, L.hidden, tok_scale);
    } else {
        const long tiles = (long)((L.n_experts + 3) / 4) * ((n_tokens + 3) / 4);
        router_logits_kernel<4, 4><<<(unsigned)((tiles + 7) / 8), 256, 0, st>>>(x, x_dtype, L.router_w, logits, n_tokens,
                                                                               L.n_experts, L.hidden, tok_scale);
    }
    if (int rc = check_launch("router_logits")) return rc;
    router_topk_kernel<<<(unsigned)((n_tokens + 7) / 8), 256, 0, st>>>(logits, L.e_bias, L.router_kind, L.renorm,
                                                                      L.routed_scaling, n_tokens, L.n_experts,
                                                                      L.top_k, ids, gates);
    return check_launch("router_topk");
}

}  // namespace chronos
