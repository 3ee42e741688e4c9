// FP4 tensor regime with the healer fused into the bank passes (layers that carry healer tiles, `ut_gu` / `ut_dn`): the
// bank-pass outputs z1 / y1 already hold the low-rank correction, so what is left between and after the passes is
// gathers, SwiGLU, the down-input transform and the gate-weighted sum - no healer product and no second read of
// healer.u_*. Mathematics as in csrc/healer_mma.cu (ChronosGlm5HolographicExpertGroup.forward_cold_fast,
// chronos_1t/models/glm5_chronos_moe.py:149-195) with the healer term already inside z1 / y1:
//   z_gu[i] = beta r_s1[i] z1[r_inv[i]];  act = silu(z_gu[:I]) z_gu[I:];  y_pair[i] = beta_d r_s1[i] y1[r_inv[i]].
#include "common.cuh"

namespace chronos {

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}

// ---------------------------------------------------------------------------------------------------------------
// Between the passes. One CTA per (work item, group of kMidGroup positions): the group's gate_up outputs (2 I floats per
// pair, bank-pass row order) are staged in shared memory; four warps per position gather the gate and up rows through
// the key table, apply SwiGLU into shared memory and sum the squares; then per pair the power-of-two scale of the down
// pass, the natural-order fp16 copy for the down healer's input factor, and the down-input transform (gather + sign,
// FWHT128, sign) quantised into the work item's FP4 image. The shared expert's rows are in natural order, no keys.
// ---------------------------------------------------------------------------------------------------------------
constexpr int kMidGroup = 4;
constexpr int kMidThreads = 512;

__global__ void __launch_bounds__(kMidThreads) mid_fused_kernel(chronos_layer_t L, Plan p) {
    extern __shared__ __align__(16) float mid_s[];  // [kMidGroup][2 I] bank-pass rows, then [kMidGroup][I] SwiGLU outputs
    __shared__ float ss_s[kMidGroup][kMidThreads / 32 / kMidGroup];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int I = L.inter, n_items = p.counters[3];
    float* zrow = mid_s;
    float* acts = mid_s + (size_t)kMidGroup * 2 * I;
    constexpr int kGroups = kPairsPerWideItem / kMidGroup, W = kMidThreads / 32 / kMidGroup;
    const int n = warp % kMidGroup, wsel = warp / kMidGroup;
    for (int w = blockIdx.x; w < n_items * kGroups; w += gridDim.x) {
        const int grp = w / n_items, item = w % n_items;
        const int start = p.gitem_start[item];
        const int cnt = min(kMidGroup, p.gitem_cnt[item] - grp * kMidGroup);
        if (cnt <= 0) continue;
        const int e = p.pair_expert[start];
        const int p0 = start + grp * kMidGroup;
        __syncthreads();  // the rows of the previous group are no longer read
        for (int u = tid; u < cnt * (2 * I / 4); u += kMidThreads) cp_async16(zrow + (size_t)u * 4, p.z1 + (size_t)p0 * 2 * I + (size_t)u * 4);
        asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncthreads();
        const bool plain = e >= L.n_experts;
        float ss = 0.0f;
        if (n < cnt) {
            const float* zn = zrow + (size_t)n * 2 * I;
            float* an = acts + (size_t)n * I;
            const float beta = plain ? 1.0f : L.gu_beta[e];
            const uint16_t* rout = L.gu_rout + (size_t)(plain ? 0 : e) * 2 * I;
            for (int i0 = (wsel * 32 + lane) * 4; i0 < I; i0 += W * 128) {
                float zg[4], zu[4];
                if (plain) {
                    const float4 a = *reinterpret_cast<const float4*>(zn + i0), b = *reinterpret_cast<const float4*>(zn + I + i0);
                    zg[0] = a.x; zg[1] = a.y; zg[2] = a.z; zg[3] = a.w;
                    zu[0] = b.x; zu[1] = b.y; zu[2] = b.z; zu[3] = b.w;
                } else {
                    const uint2 rg = *reinterpret_cast<const uint2*>(rout + i0), ru = *reinterpret_cast<const uint2*>(rout + I + i0);
                    const uint32_t eg[4] = {rg.x & 0xffffu, rg.x >> 16, rg.y & 0xffffu, rg.y >> 16};
                    const uint32_t eu[4] = {ru.x & 0xffffu, ru.x >> 16, ru.y & 0xffffu, ru.y >> 16};
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float vg = zn[eg[q] & 0x7fffu], vu = zn[eu[q] & 0x7fffu];
                        zg[q] = beta * ((eg[q] >> 15) ? -vg : vg);
                        zu[q] = beta * ((eu[q] >> 15) ? -vu : vu);
                    }
                }
                if (p.tail_gu != nullptr && !plain) {
                    const float4 tg = *reinterpret_cast<const float4*>(p.tail_gu + (size_t)(p0 + n) * 2 * I + i0);
                    const float4 tu = *reinterpret_cast<const float4*>(p.tail_gu + (size_t)(p0 + n) * 2 * I + I + i0);
                    zg[0] += tg.x; zg[1] += tg.y; zg[2] += tg.z; zg[3] += tg.w;
                    zu[0] += tu.x; zu[1] += tu.y; zu[2] += tu.z; zu[3] += tu.w;
                }
                float a[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    a[q] = silu_f32(zg[q]) * zu[q];
                    ss = fmaf(a[q], a[q], ss);
                }
                *reinterpret_cast<float4*>(an + i0) = make_float4(a[0], a[1], a[2], a[3]);
            }
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        if (lane == 0) ss_s[n][wsel] = ss;
        __syncthreads();
        if (n < cnt) {
            float tot = 0.0f;
#pragma unroll
            for (int q = 0; q < W; ++q) tot += ss_s[n][q];
            const float gsc = pow2_scale(tot, I), gi = 1.0f / gsc;
            const int pos = grp * kMidGroup + n, pair = p0 + n;
            const float* an = acts + (size_t)n * I;
            if (wsel == 0 && lane == 0) p.pscale_dn[pair] = gsc;
            // a warp takes a whole 256-column stage: its two half-warps each transform one 128-block, eight values per lane
            const int half = lane >> 4, jl = lane & 15;
            const uint16_t* cin = L.dn_cin + (size_t)(plain ? 0 : e) * I + half * 128 + jl * 8;
            const uint32_t* cs2 = L.dn_cs2 + (size_t)(plain ? 0 : e) * (I / 32) + half * 4 + (jl >> 2);
            uint8_t* img0 = p.bq_dn + (size_t)item * (I / 256) * kWideStageBytes;
            for (int st = wsel; st < I / 256; st += W) {
                const int k0 = st * 256 + half * 128 + jl * 8;
                const float4 a0 = *reinterpret_cast<const float4*>(an + k0), a1 = *reinterpret_cast<const float4*>(an + k0 + 4);
                const float s8[8] = {a0.x * gi, a0.y * gi, a0.z * gi, a0.w * gi, a1.x * gi, a1.y * gi, a1.z * gi, a1.w * gi};
                {   // natural order, for V_down . act
                    const float lo4[4] = {s8[0], s8[1], s8[2], s8[3]}, hi4[4] = {s8[4], s8[5], s8[6], s8[7]};
                    store_half4(p.ac + (size_t)pair * I + k0, lo4);
                    store_half4(p.ac + (size_t)pair * I + k0 + 4, hi4);
                }
                float v[8];
                if (plain) {
#pragma unroll
                    for (int q = 0; q < 8; ++q) v[q] = s8[q];
                } else {
                    const uint4 ce = *reinterpret_cast<const uint4*>(cin + st * 256);
                    const uint32_t ent[8] = {ce.x & 0xffffu, ce.x >> 16, ce.y & 0xffffu, ce.y >> 16,
                                             ce.z & 0xffffu, ce.z >> 16, ce.w & 0xffffu, ce.w >> 16};
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const float av = an[ent[q] & 0x7fffu];
                        v[q] = (ent[q] >> 15) ? -av : av;
                    }
                    fwht128_half(v, lane);
                    const uint32_t sw = cs2[st * 8] >> ((jl & 3) * 8);
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        if ((sw >> q) & 1u) v[q] = -v[q];
                        v[q] *= gi;
                    }
                }
                quantize_stage_fp4x3<kWideRows, kPairsPerWideItem>(v, lane, img0 + (size_t)st * kWideStageBytes, pos);
            }
        }
    }
}

int launch_mid_fused(const chronos_layer_t& L, const Plan& p, cudaStream_t st) {
    const size_t smem = (size_t)kMidGroup * 3 * L.inter * 4;
    if (int rc = ensure_dynamic_smem(reinterpret_cast<const void*>(mid_fused_kernel), smem, "mid_fused")) return rc;
    const long most = (long)p.max_gitems * (kPairsPerWideItem / kMidGroup);
    const long resident = (long)device_sm_count() * (smem * 3 <= 200 * 1024 ? 3 : (smem * 2 <= 200 * 1024 ? 2 : 1));
    mid_fused_kernel<<<(unsigned)(most < resident ? most : resident), kMidThreads, smem, st>>>(L, p);
    return check_launch("mid_fused");
}

// ---------------------------------------------------------------------------------------------------------------
// After the down pass: y[t, i] = sum_j gate[t, j] * (beta_d r_s1[i] y1[pos(t, j)][r_inv[i]]) (+ the shared expert's row),
// j in index order. One CTA per token at a time: the token's rows (bank-pass row order, H floats each) are staged in
// shared memory kCgRows at a time, so the gathers through the key tables cost shared-memory reads; every thread keeps
// the running sums of its output columns in registers across the stagings. Two CTAs per SM overlap each other's copies.
// ---------------------------------------------------------------------------------------------------------------
constexpr int kCgRows = 5;
constexpr int kCgThreads = 512;
constexpr int kCgMaxGroups = 4;   // output columns per thread = 4 * groups: hidden <= 4 * 4 * 512 = 8192
constexpr int kCgMaxEntries = 40; // top_k (<= 32) + the shared expert, rounded up

__global__ void __launch_bounds__(kCgThreads) combine_gather_kernel(chronos_layer_t L, Plan p, const float* __restrict__ gates,
                                                                    int n_tokens, int with_shared, void* __restrict__ y, int y_dtype) {
    extern __shared__ __align__(16) float cg_rows[];  // [kCgRows][H]
    __shared__ int e_pos[kCgMaxEntries], e_exp[kCgMaxEntries];
    __shared__ float e_gate[kCgMaxEntries], e_beta[kCgMaxEntries];
    const int tid = threadIdx.x;
    const int H = L.hidden, k = L.top_k;
    const int n_groups = (H + kCgThreads * 4 - 1) / (kCgThreads * 4);
    for (int t = blockIdx.x; t < n_tokens; t += gridDim.x) {
        const bool shared_row = with_shared && t >= p.shared_lo && t < p.shared_lo + p.shared_n;
        const int n_ent = k + (shared_row ? 1 : 0);
        __syncthreads();  // the entry table and the rows of the previous token are no longer read
        if (tid < n_ent) {
            int pos, e = L.n_experts;
            float g = 1.0f, beta = 1.0f;
            if (tid < k) {
                pos = p.pos_of[t * k + tid];
                if (pos >= 0) { e = p.pair_expert[pos]; g = gates[t * k + tid]; beta = L.dn_beta[e]; }
            } else {
                pos = p.offsets[L.n_experts] + t - p.shared_lo;
            }
            e_pos[tid] = pos; e_exp[tid] = e; e_gate[tid] = g; e_beta[tid] = beta;
        }
        __syncthreads();
        float acc[kCgMaxGroups][4];
#pragma unroll
        for (int gI = 0; gI < kCgMaxGroups; ++gI)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[gI][q] = 0.0f;
        for (int base = 0; base < n_ent; base += kCgRows) {
            if (base > 0) __syncthreads();  // the previous staging has been summed
            const int rows_here = min(kCgRows, n_ent - base);
            for (int jj = 0; jj < rows_here; ++jj) {  // row by row: no division in the copy loop
                const int pos = e_pos[base + jj];
                if (pos < 0) continue;
                const float* src = p.y1 + (size_t)pos * H;
                float* dst = cg_rows + (size_t)jj * H;
                for (int c = tid * 4; c < H; c += kCgThreads * 4) cp_async16(dst + c, src + c);
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
            asm volatile("cp.async.wait_all;" ::: "memory");
            __syncthreads();
            for (int jj = 0; jj < rows_here; ++jj) {
                const int pos = e_pos[base + jj];
                if (pos < 0) continue;  // block-uniform
                const int e = e_exp[base + jj];
                const float g = e_gate[base + jj], beta = e_beta[base + jj];
                const float* row = cg_rows + (size_t)jj * H;
                const bool plain = e >= L.n_experts;
                const bool tail = p.tail_dn != nullptr && !plain;
                const float gb = g * beta;  // without a tail term the two factors of a routed entry are applied as one
                const uint16_t* rout = L.dn_rout + (size_t)(plain ? 0 : e) * H;
#pragma unroll
                for (int gI = 0; gI < kCgMaxGroups; ++gI) {
                    const int i0 = (gI * kCgThreads + tid) * 4;
                    if (gI >= n_groups || i0 >= H) break;
                    float v[4];
                    if (plain) {
                        const float4 r4 = *reinterpret_cast<const float4*>(row + i0);
                        v[0] = r4.x; v[1] = r4.y; v[2] = r4.z; v[3] = r4.w;
                    } else {
                        const uint2 r2 = *reinterpret_cast<const uint2*>(rout + i0);
                        const uint32_t ent[4] = {r2.x & 0xffffu, r2.x >> 16, r2.y & 0xffffu, r2.y >> 16};
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const float yv = row[ent[q] & 0x7fffu];
                            v[q] = (ent[q] >> 15) ? -yv : yv;
                        }
                    }
                    if (plain) {
#pragma unroll
                        for (int q = 0; q < 4; ++q) acc[gI][q] += v[q];
                    } else if (tail) {
                        const float4 t4 = *reinterpret_cast<const float4*>(p.tail_dn + (size_t)pos * H + i0);
                        const float tl[4] = {t4.x, t4.y, t4.z, t4.w};
#pragma unroll
                        for (int q = 0; q < 4; ++q) acc[gI][q] = fmaf(g, fmaf(beta, v[q], tl[q]), acc[gI][q]);
                    } else {
#pragma unroll
                        for (int q = 0; q < 4; ++q) acc[gI][q] = fmaf(gb, v[q], acc[gI][q]);
                    }
                }
            }
        }
#pragma unroll
        for (int gI = 0; gI < kCgMaxGroups; ++gI) {
            const int i0 = (gI * kCgThreads + tid) * 4;
            if (gI >= n_groups || i0 >= H) break;
            if (y_dtype == CHRONOS_DTYPE_BF16) {
                __nv_bfloat162 a01 = __floats2bfloat162_rn(acc[gI][0], acc[gI][1]), a23 = __floats2bfloat162_rn(acc[gI][2], acc[gI][3]);
                uint2 o;
                o.x = *reinterpret_cast<uint32_t*>(&a01);
                o.y = *reinterpret_cast<uint32_t*>(&a23);
                *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(y) + (size_t)t * H + i0) = o;
            } else {
                *reinterpret_cast<float4*>(reinterpret_cast<float*>(y) + (size_t)t * H + i0) = make_float4(acc[gI][0], acc[gI][1], acc[gI][2], acc[gI][3]);
            }
        }
    }
}

bool combine_gather_fits(const chronos_layer_t& L) {
    return L.hidden <= kCgMaxGroups * kCgThreads * 4 && L.top_k + 1 <= kCgMaxEntries && (size_t)kCgRows * L.hidden * 4 <= 200 * 1024;
}

int launch_combine_gather(const chronos_layer_t& L, const Plan& p, const float* gates, int n_tokens, int with_shared, void* y,
                          int y_dtype, cudaStream_t st) {
    if (n_tokens <= 0) return CHRONOS_OK;
    const size_t smem = (size_t)kCgRows * L.hidden * 4;
    if (int rc = ensure_dynamic_smem(reinterpret_cast<const void*>(combine_gather_kernel), smem, "combine_gather")) return rc;
    const int resident = device_sm_count() * (smem * 2 <= 200 * 1024 ? 2 : 1);
    combine_gather_kernel<<<(unsigned)(n_tokens < resident ? n_tokens : resident), kCgThreads, smem, st>>>(
        L, p, gates, n_tokens, with_shared && L.shared_inter > 0, y, y_dtype);
    return check_launch("combine_gather");
}

}  // namespace chronos
