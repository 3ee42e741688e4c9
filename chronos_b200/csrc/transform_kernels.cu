// Activation-space unfold around the two bank passes: the per-expert sign / permutation / 128-block Hadamard
// transforms, the rank-r healer factors, SwiGLU and the gate-weighted combine. Mathematics of
// ChronosGlm5HolographicExpertGroup.forward_cold_fast (chronos_1t/models/glm5_chronos_moe.py:149-195):
//   x_c = c_s2 * H((x * c_s1)[c_perm]);  z = r_s1 * H(r_s2 * (S x_c))[r_inv];  z_gu = beta z + U (V x)
//   act = silu(z_gu[:I]) * z_gu[I:];     same transform for down;  y += gate * (beta_d z_d + U_d (V_d act))
#include "common.cuh"

namespace chronos {

// ---------------------------------------------------------------------------------------------------------------
// gate_up input: one warp per (sorted pair, 128-column block) writes x_c in fp16; further warps compute V_gu . x.
// ---------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) pre_gu_kernel(chronos_layer_t L, const void* __restrict__ x, int x_dtype, Plan p) {
    const int lane = threadIdx.x & 31;
    const long gw = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int n_pairs = p.counters[1];
    const int H = L.hidden, E = L.n_experts, r = L.rank;
    const int nblk = H / 128;
    const long xf_warps = (long)p.max_pairs * nblk;
    if (gw < xf_warps) {
        const int pair = (int)(gw / nblk), blk = (int)(gw % nblk);
        if (pair >= n_pairs) return;
        const int t = p.pair_token[pair], e = p.pair_expert[pair];
        float v[4];
        if (e >= E) {  // shared expert: plain weights, identity keys
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = ld_act(x, x_dtype, (size_t)t * H + blk * 128 + lane * 4 + i);
        } else {
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
        __half2 h01 = __halves2half2(f32_to_f16_sat(v[0]), f32_to_f16_sat(v[1]));
        __half2 h23 = __halves2half2(f32_to_f16_sat(v[2]), f32_to_f16_sat(v[3]));
        uint2 o;
        o.x = *reinterpret_cast<uint32_t*>(&h01);
        o.y = *reinterpret_cast<uint32_t*>(&h23);
        *reinterpret_cast<uint2*>(p.xc + (size_t)pair * H + blk * 128 + lane * 4) = o;
        return;
    }
    // healer input factor: hmid[pair, c] = sum_k V_gu[e, c, k] * x[t, k]; one warp per (pair, 8 rank rows).
    // Lane l owns 16 consecutive columns per 512-column step: one 16-byte load per rank row.
    const long hw = gw - xf_warps;
    const int rgroups = r / 8;
    const int pair = (int)(hw / rgroups), rg = (int)(hw % rgroups);
    if (pair >= n_pairs) return;
    const int t = p.pair_token[pair], e = p.pair_expert[pair];
    if (e >= E) return;
    float acc[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] = 0.0f;
    const uint8_t* vbase = L.v_gu + ((size_t)e * r + rg * 8) * H;
    for (int k = lane * 16; k < H; k += 512) {
        uint4 vw[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) vw[c] = *reinterpret_cast<const uint4*>(vbase + (size_t)c * H + k);
        float xv[16];
        ld_act16(x, x_dtype, (size_t)t * H + k, xv);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const uint32_t ww[4] = {vw[c].x, vw[c].y, vw[c].z, vw[c].w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float2 lo = e4m3x2_to_f32((uint16_t)(ww[q] & 0xffffu)), hi = e4m3x2_to_f32((uint16_t)(ww[q] >> 16));
                acc[c] = fmaf(lo.x, xv[q * 4 + 0], acc[c]);
                acc[c] = fmaf(lo.y, xv[q * 4 + 1], acc[c]);
                acc[c] = fmaf(hi.x, xv[q * 4 + 2], acc[c]);
                acc[c] = fmaf(hi.y, xv[q * 4 + 3], acc[c]);
            }
        }
    }
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        float s = acc[c];
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        if (lane == 0) p.hmid[(size_t)pair * r + rg * 8 + c] = s;
    }
}

int launch_pre_gu(const chronos_layer_t& L, const void* x, int x_dtype, const Plan& p, cudaStream_t st) {
    const long warps = (long)p.max_pairs * (L.hidden / 128) + (long)p.max_pairs * (L.rank / 8);
    pre_gu_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(L, x, x_dtype, p);
    return check_launch("pre_gu");
}

// ---------------------------------------------------------------------------------------------------------------
// Between the passes: one warp per (sorted pair, 128-block of the down input). Each down-input element needs one
// SwiGLU output, which needs two gate_up rows (row-inverse gather of z1 + beta + healer U_gu . hmid).
// ---------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) mid_kernel(chronos_layer_t L, Plan p) {
    __shared__ float hs[8][kMaxRank];
    __shared__ float act_s[8][128];
    __shared__ uint16_t idx_s[8][128];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const long gw = (long)blockIdx.x * 8 + wib;
    const int n_pairs = p.counters[1];
    const int H = L.hidden, I = L.inter, E = L.n_experts, r = L.rank;
    const int nblk = I / 128;
    const int pair = (int)(gw / nblk), blk = (int)(gw % nblk);
    if (pair >= n_pairs) return;
    const int e = p.pair_expert[pair];
    const float* z1 = p.z1 + (size_t)pair * 2 * I;
    __half* ac = p.ac + (size_t)pair * I + blk * 128 + lane * 4;
    float v[4];
    if (e >= E) {  // shared expert: rows in natural order, no healer
        const float4 zg = *reinterpret_cast<const float4*>(z1 + blk * 128 + lane * 4);
        const float4 zu = *reinterpret_cast<const float4*>(z1 + I + blk * 128 + lane * 4);
        v[0] = silu_f32(zg.x) * zu.x; v[1] = silu_f32(zg.y) * zu.y;
        v[2] = silu_f32(zg.z) * zu.z; v[3] = silu_f32(zg.w) * zu.w;
    } else {
        for (int c = lane; c < r; c += 32) hs[wib][c] = p.hmid[(size_t)pair * r + c];
        __syncwarp();
        const float beta = L.gu_beta[e];
        const uint2 ce = *reinterpret_cast<const uint2*>(L.dn_cin + (size_t)e * I + blk * 128 + lane * 4);
        const uint32_t ent[4] = {ce.x & 0xffffu, ce.x >> 16, ce.y & 0xffffu, ce.y >> 16};
        const uint16_t* rout = L.gu_rout + (size_t)e * 2 * I;
        const uint8_t* ug = L.u_gu + (size_t)e * 2 * I * r;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int src_i = (int)(ent[i] & 0x7fffu);  // SwiGLU index feeding down-input position j
            float zz[2];
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int row = src_i + half * I;
                const uint16_t ro = rout[row];
                float zb = z1[ro & 0x7fff];
                if (ro >> 15) zb = -zb;
                float heal = 0.0f;
                const uint4* urow = reinterpret_cast<const uint4*>(ug + (size_t)row * r);
                for (int c16 = 0; c16 < r / 16; ++c16) {
                    const uint4 u = urow[c16];
                    const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float2 lo = e4m3x2_to_f32((uint16_t)(uw[q] & 0xffffu));
                        const float2 hi = e4m3x2_to_f32((uint16_t)(uw[q] >> 16));
                        const float* hp = &hs[wib][c16 * 16 + q * 4];
                        heal = fmaf(lo.x, hp[0], heal);
                        heal = fmaf(lo.y, hp[1], heal);
                        heal = fmaf(hi.x, hp[2], heal);
                        heal = fmaf(hi.y, hp[3], heal);
                    }
                }
                zz[half] = fmaf(beta, zb, heal);
            }
            const float a = silu_f32(zz[0]) * zz[1];
            act_s[wib][lane * 4 + i] = a;
            idx_s[wib][lane * 4 + i] = (uint16_t)src_i;
            v[i] = (ent[i] >> 15) ? -a : a;
        }
        fwht128_warp(v, lane);
        const uint32_t sw = L.dn_cs2[(size_t)e * (I / 32) + blk * 4 + lane / 8] >> ((lane & 7) * 4);
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if ((sw >> i) & 1u) v[i] = -v[i];
        __syncwarp();
        // partial down-healer input: hpart[pair, blk, c] = sum_{j in block} V_down^T[e, i(j), c] * act(i(j)).
        // A row of V_down^T is r bytes = r/16 chunks of 16; lane = (row selector, chunk): 32/(r/16) rows per step.
        const uint8_t* vt = L.v_dn_t + (size_t)e * I * r;
        const int cpr = r / 16, rpi = 32 / cpr;
        const int rsel = lane / cpr, chunk = lane % cpr;
        float hacc[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) hacc[c] = 0.0f;
#pragma unroll 4
        for (int j0 = 0; j0 < 128; j0 += rpi) {
            const int jj = j0 + rsel;
            const uint4 w = *reinterpret_cast<const uint4*>(vt + (size_t)idx_s[wib][jj] * r + chunk * 16);
            const float a = act_s[wib][jj];
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float2 lo = e4m3x2_to_f32((uint16_t)(ww[q] & 0xffffu)), hi = e4m3x2_to_f32((uint16_t)(ww[q] >> 16));
                hacc[q * 4 + 0] = fmaf(lo.x, a, hacc[q * 4 + 0]);
                hacc[q * 4 + 1] = fmaf(lo.y, a, hacc[q * 4 + 1]);
                hacc[q * 4 + 2] = fmaf(hi.x, a, hacc[q * 4 + 2]);
                hacc[q * 4 + 3] = fmaf(hi.y, a, hacc[q * 4 + 3]);
            }
        }
        for (int off = cpr; off < 32; off <<= 1)
#pragma unroll
            for (int c = 0; c < 16; ++c) hacc[c] += __shfl_xor_sync(0xffffffffu, hacc[c], off);
        if (rsel == 0) {
            float4* hp = reinterpret_cast<float4*>(p.hpart + ((size_t)pair * nblk + blk) * r + chunk * 16);
#pragma unroll
            for (int q = 0; q < 4; ++q) hp[q] = make_float4(hacc[q * 4], hacc[q * 4 + 1], hacc[q * 4 + 2], hacc[q * 4 + 3]);
        }
    }
    __half2 h01 = __halves2half2(f32_to_f16_sat(v[0]), f32_to_f16_sat(v[1]));
    __half2 h23 = __halves2half2(f32_to_f16_sat(v[2]), f32_to_f16_sat(v[3]));
    uint2 o;
    o.x = *reinterpret_cast<uint32_t*>(&h01);
    o.y = *reinterpret_cast<uint32_t*>(&h23);
    *reinterpret_cast<uint2*>(ac) = o;
    (void)H;
}

int launch_mid(const chronos_layer_t& L, const Plan& p, cudaStream_t st) {
    const long warps = (long)p.max_pairs * (L.inter / 128);
    mid_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(L, p);
    return check_launch("mid");
}

// ---------------------------------------------------------------------------------------------------------------
// Combine: y[t, i] = sum_j gate[t, j] * (beta_d * r_s1[i] * y1[p_j, r_inv[i]] + U_down[e_j, i, :] . hd[p_j, :])
//                    (+ shared expert row), summed over j = 0..top_k-1 in that order.
// One block per (token, 128 output rows): warp w evaluates routing entries j = w, w+8, ...; lane l owns rows 4l..4l+3;
// the per-entry terms meet in shared memory and are added in index order (deterministic).
// ---------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) combine_kernel(chronos_layer_t L, Plan p, const float* __restrict__ gates,
                                                      int with_shared, void* __restrict__ y, int y_dtype) {
    __shared__ float hd[8][kMaxRank];
    __shared__ __align__(16) float terms[kMaxTopK][128];
    const int t = blockIdx.x, rb = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int H = L.hidden, I = L.inter, E = L.n_experts, r = L.rank, k = L.top_k;
    const int nblk = I / 128;
    const int row0 = rb * 128 + lane * 4;
    for (int j = warp; j < k; j += 8) {
        const int pos = p.pos_of[t * k + j];
        float out[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (pos >= 0) {
            for (int c = lane; c < r; c += 32) {
                float s = 0.0f;
                for (int b = 0; b < nblk; ++b) s += p.hpart[((size_t)pos * nblk + b) * r + c];
                hd[warp][c] = s;
            }
            __syncwarp();
            const int e = p.pair_expert[pos];
            const float g = gates[t * k + j], beta = L.dn_beta[e];
            const uint2 ro2 = *reinterpret_cast<const uint2*>(L.dn_rout + (size_t)e * H + row0);
            const uint32_t ro[4] = {ro2.x & 0xffffu, ro2.x >> 16, ro2.y & 0xffffu, ro2.y >> 16};
            float yb[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float v = p.y1[(size_t)pos * H + (ro[q] & 0x7fffu)];
                yb[q] = (ro[q] >> 15) ? -v : v;
            }
            const uint4* urow = reinterpret_cast<const uint4*>(L.u_dn + ((size_t)e * H + row0) * r);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                float heal = 0.0f;
                for (int c16 = 0; c16 < r / 16; ++c16) {
                    const uint4 u = urow[q * (r / 16) + c16];
                    const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                    for (int w4 = 0; w4 < 4; ++w4) {
                        const float2 lo = e4m3x2_to_f32((uint16_t)(uw[w4] & 0xffffu));
                        const float2 hi = e4m3x2_to_f32((uint16_t)(uw[w4] >> 16));
                        const float* hp = &hd[warp][c16 * 16 + w4 * 4];
                        heal = fmaf(lo.x, hp[0], heal);
                        heal = fmaf(lo.y, hp[1], heal);
                        heal = fmaf(hi.x, hp[2], heal);
                        heal = fmaf(hi.y, hp[3], heal);
                    }
                }
                out[q] = g * fmaf(beta, yb[q], heal);
            }
            __syncwarp();
        }
        *reinterpret_cast<float4*>(&terms[j][lane * 4]) = make_float4(out[0], out[1], out[2], out[3]);
    }
    __syncthreads();
    if (threadIdx.x < 128) {
        const int i = rb * 128 + threadIdx.x;
        float acc = 0.0f;
        for (int j = 0; j < k; ++j) acc += terms[j][threadIdx.x];
        if (with_shared) acc += p.y1[(size_t)(p.offsets[E] + t) * H + i];
        if (y_dtype == CHRONOS_DTYPE_BF16)
            reinterpret_cast<__nv_bfloat16*>(y)[(size_t)t * H + i] = __float2bfloat16(acc);
        else
            reinterpret_cast<float*>(y)[(size_t)t * H + i] = acc;
    }
}

int launch_combine(const chronos_layer_t& L, const Plan& p, const float* gates, int n_tokens, int with_shared, void* y,
                   int y_dtype, cudaStream_t st) {
    if (n_tokens <= 0) return CHRONOS_OK;
    dim3 grid((unsigned)n_tokens, (unsigned)(L.hidden / 128));
    combine_kernel<<<grid, 256, 0, st>>>(L, p, gates, with_shared && L.shared_inter > 0, y, y_dtype);
    return check_launch("combine");
}

// ---------------------------------------------------------------------------------------------------------------
// Residual add + RMSNorm (chronos_1t/models/glm53_engine.py:71-73, :203): one block per token, fp32 math.
// ---------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) residual_rmsnorm_kernel(void* __restrict__ h, const void* __restrict__ y,
                                                               const float* __restrict__ w, void* __restrict__ xn,
                                                               int dtype, int hidden, float eps) {
    __shared__ float red[8];
    const size_t base = (size_t)blockIdx.x * hidden;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < hidden; i += 256) {
        float v = ld_act(h, dtype, base + i);
        if (y) {
            v += ld_act(y, dtype, base + i);
            if (dtype == CHRONOS_DTYPE_BF16) {
                const __nv_bfloat16 b = __float2bfloat16(v);
                reinterpret_cast<__nv_bfloat16*>(h)[base + i] = b;
                v = __bfloat162float(b);
            } else {
                reinterpret_cast<float*>(h)[base + i] = v;
            }
        }
        ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int q = 0; q < 8; ++q) tot += red[q];
    const float inv = rsqrtf(tot / (float)hidden + eps);
    for (int i = threadIdx.x; i < hidden; i += 256) {
        float v = ld_act(h, dtype, base + i) * inv;
        if (w) v *= w[i];
        if (dtype == CHRONOS_DTYPE_BF16)
            reinterpret_cast<__nv_bfloat16*>(xn)[base + i] = __float2bfloat16(v);
        else
            reinterpret_cast<float*>(xn)[base + i] = v;
    }
}

int launch_residual_rmsnorm(void* h, const void* y, const float* w, void* xn, int dtype, int n_tokens, int hidden,
                            float eps, cudaStream_t st) {
    if (n_tokens <= 0) return CHRONOS_OK;
    residual_rmsnorm_kernel<<<(unsigned)n_tokens, 256, 0, st>>>(h, y, w, xn, dtype, hidden, eps);
    return check_launch("residual_rmsnorm");
}

}  // namespace chronos
