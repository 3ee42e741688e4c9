// Activation-space unfold around the two bank passes: the per-expert sign / permutation / 128-block Hadamard
// transforms, the rank-r healer factors, SwiGLU and the gate-weighted combine. Mathematics of
// ChronosGlm5HolographicExpertGroup.forward_cold_fast (chronos_1t/models/glm5_chronos_moe.py:149-195):
//   x_c = c_s2 * H((x * c_s1)[c_perm]);  z = r_s1 * H(r_s2 * (S x_c))[r_inv];  z_gu = beta z + U (V x)
//   act = silu(z_gu[:I]) * z_gu[I:];     same transform for down;  y += gate * (beta_d z_d + U_d (V_d act))
#include "common.cuh"

namespace chronos {


// ---------------------------------------------------------------------------------------------------------------
// gate_up input. Transform warps: fp16 mode - one warp per (sorted pair, 128-column block) writes x_c;
// FP4 mode - one warp per (work item, position in item, 128-column block) writes three e2m1 terms into the item's
// activation image (positions past the item's pair count stay unwritten). Further warps compute V_gu . x.
// ---------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) pre_gu_kernel(chronos_layer_t L, const void* __restrict__ x, int x_dtype, Plan p,
                                                     int fp4) {
    const int lane = threadIdx.x & 31;
    const long gw = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int n_pairs = p.counters[1];
    const int H = L.hidden, E = L.n_experts, r = L.rank;
    const int nblk = H / 128;
    const long xf_warps = fp4 ? (long)p.max_items * kPairsPerItem * nblk : (long)p.max_pairs * nblk;
    if (gw < xf_warps) {
        float v[4];
        if (!fp4) {
            const int pair = (int)(gw / nblk), blk = (int)(gw % nblk);
            if (pair >= n_pairs) return;
            const int t = p.pair_token[pair];
            const float g = p.tok_scale[t];  // power of two: keeps the fp16 image in range whatever the activation scale
            transform_gu_block(L, x, x_dtype, t, p.pair_expert[pair], blk, lane, v);
            const float gi = 1.0f / g;
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] *= gi;
            if (blk == 0 && lane == 0) p.pscale_gu[pair] = g;
            store_half4(p.xc + (size_t)pair * H + blk * 128 + lane * 4, v);
            return;
        }
        const int blk = (int)(gw % nblk);
        const int ip = (int)(gw / nblk), item = ip / kPairsPerItem, pos = ip % kPairsPerItem;
        // positions past the item's pair count are left unwritten: row n of the image only feeds accumulator column n,
        // and the bank pass never reads the columns of absent pairs
        if (item >= p.counters[0] || pos >= p.item_cnt[item]) return;
        {
            const int pair = p.item_start[item] + pos;
            const int t = p.pair_token[pair];
            const float g = p.tok_scale[t];
            transform_gu_block(L, x, x_dtype, t, p.pair_expert[pair], blk, lane, v);
            const float gi = 1.0f / g;
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] *= gi;
            if (blk == 0 && lane == 0) p.pscale_gu[pair] = g;
        }
        uint8_t* img = p.bq_gu + ((size_t)item * (H / 256) + blk / 2) * 6144;
        quantize_block_fp4x3<32, 8>(v, lane, img, blk & 1, pos);
        return;
    }
    // healer input factor: hmid[pair, c] = sum_k V_gu[e, c, k] * x[t, k]; one warp per (pair, rank row): the row's
    // 16-byte pieces (lane l owns columns 16 l .. 16 l + 15 of every 512-column step) are all requested before use.
    const long hw = gw - xf_warps;
    const int pair = (int)(hw / r), c = (int)(hw % r);
    if (pair >= n_pairs) return;
    const int t = p.pair_token[pair], e = p.pair_expert[pair];
    if (e >= E) return;
    const uint8_t* vrow = L.v_gu + ((size_t)e * r + c) * H;
    float acc = 0.0f;
    for (int k0 = 0; k0 < H; k0 += 4 * 512) {
        uint4 vw[4];
        float xv[4][16];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int k = k0 + u * 512 + lane * 16;
            if (k < H) vw[u] = *reinterpret_cast<const uint4*>(vrow + k);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int k = k0 + u * 512 + lane * 16;
            if (k < H) ld_act16(x, x_dtype, (size_t)t * H + k, xv[u]);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int k = k0 + u * 512 + lane * 16;
            if (k < H) {
                const uint32_t ww[4] = {vw[u].x, vw[u].y, vw[u].z, vw[u].w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float2 lo = e4m3x2_to_f32((uint16_t)(ww[q] & 0xffffu)), hi = e4m3x2_to_f32((uint16_t)(ww[q] >> 16));
                    acc = fmaf(lo.x, xv[u][q * 4 + 0], acc);
                    acc = fmaf(lo.y, xv[u][q * 4 + 1], acc);
                    acc = fmaf(hi.x, xv[u][q * 4 + 2], acc);
                    acc = fmaf(hi.y, xv[u][q * 4 + 3], acc);
                }
            }
        }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) p.hmid[(size_t)pair * r + c] = acc;
}

// Healer input factor for batches with many pairs per expert: a block = 8 consecutive sorted pairs x 8 rank rows; warp w
// computes the 8 dots of pair 8 b + w, and the 8 warps share the 8 rows of V_gu through L1 when they share the expert.
__global__ void __launch_bounds__(256) healer_in_tile_kernel(chronos_layer_t L, const void* __restrict__ x, int x_dtype, Plan p) {
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int H = L.hidden, r = L.rank, rgroups = r / 8;
    const int pair = (int)(blockIdx.x / rgroups) * 8 + wib, rg = (int)(blockIdx.x % rgroups);
    if (pair >= p.counters[1]) return;
    const int t = p.pair_token[pair], e = p.pair_expert[pair];
    if (e >= L.n_experts) return;
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
        float sacc = acc[c];
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) sacc += __shfl_xor_sync(0xffffffffu, sacc, off);
        if (lane == 0) p.hmid[(size_t)pair * r + rg * 8 + c] = sacc;
    }
}

// Per-token power-of-two scale near rms(x[t]); one warp per token, fixed summation order.
__global__ void __launch_bounds__(256) token_scale_kernel(const void* __restrict__ x, int x_dtype, int n_tokens, int hidden,
                                                          float* __restrict__ tok_scale) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (t >= n_tokens) return;
    float ss = 0.0f;
    if (hidden % 512 == 0) {  // 16 consecutive elements per lane and step (vector loads); the order is fixed all the same
        for (int k = lane * 16; k < hidden; k += 512) {
            float v[16];
            ld_act16(x, x_dtype, (size_t)t * hidden + k, v);
#pragma unroll
            for (int i = 0; i < 16; ++i) ss = fmaf(v[i], v[i], ss);
        }
    } else {
        for (int k = lane; k < hidden; k += 32) {
            const float v = ld_act(x, x_dtype, (size_t)t * hidden + k);
            ss = fmaf(v, v, ss);
        }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) tok_scale[t] = pow2_scale(ss, hidden);
}

// x / token scale as fp16 rows: the activation source of the large-batch kernels (read many times per token).
__global__ void __launch_bounds__(256) tokens_f16_kernel(const void* __restrict__ x, int x_dtype, long n_elems, int hidden,
                                                         const float* __restrict__ tok_scale, __half* __restrict__ x16) {
    const long i = ((long)blockIdx.x * 256 + threadIdx.x) * 4;
    if (i >= n_elems) return;
    const float gi = 1.0f / tok_scale[i / hidden];
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = ld_act(x, x_dtype, (size_t)i + j) * gi;
    store_half4(x16 + i, v);
}

int launch_tokens_f16(const void* x, int x_dtype, int n_tokens, int hidden, const float* tok_scale, __half* x16, cudaStream_t st) {
    const long n = (long)n_tokens * hidden;
    tokens_f16_kernel<<<(unsigned)((n / 4 + 255) / 256), 256, 0, st>>>(x, x_dtype, n, hidden, tok_scale, x16);
    return check_launch("tokens_f16");
}

int launch_token_scale(const void* x, int x_dtype, int n_tokens, int hidden, float* tok_scale, cudaStream_t st) {
    if (n_tokens <= 0) return CHRONOS_OK;
    token_scale_kernel<<<(unsigned)((n_tokens + 7) / 8), 256, 0, st>>>(x, x_dtype, n_tokens, hidden, tok_scale);
    return check_launch("token_scale");
}

// FP4 tensor regime: the activation images of a work item (up to 64 pairs of one expert; per 256-column stage 192 rows =
// 3 residual terms x 64 positions). One CTA per (work item, group of kPreGuGroup positions): the group's token rows
// (fp16, already divided by the token scale) are staged in shared memory by asynchronous copies, so that the gather of
// the key permutation - which reaches anywhere in the row - costs shared-memory reads instead of one L1 sector per
// element; warp tasks = (position, 128-block): gather + sign, FWHT, sign, three FP4 terms written straight into the
// image (2 bytes per lane; the positions of a group fill each 16-byte row unit's neighbours, so the sectors merge in L2).
// Rows of absent positions are not written: their MMA columns are never read back.
constexpr int kPreGuGroup = 4;
constexpr int kPreGuThreads = 512;

__global__ void __launch_bounds__(kPreGuThreads) pre_gu_wide_kernel(chronos_layer_t L, Plan p) {
    extern __shared__ __align__(16) __half rows_s[];  // [kPreGuGroup][hidden]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int H = L.hidden, n_items = p.counters[3];
    constexpr int kGroups = kPairsPerWideItem / kPreGuGroup;
    for (int w = blockIdx.x; w < n_items * kGroups; w += gridDim.x) {
        const int grp = w / n_items, item = w % n_items;  // item fastest: neighbouring CTAs get comparable work
        const int start = p.gitem_start[item];
        const int cnt = min(kPreGuGroup, p.gitem_cnt[item] - grp * kPreGuGroup);
        if (cnt <= 0) continue;
        const int e = p.pair_expert[start];
        __syncthreads();  // the rows of the previous group are no longer read
        for (int n = 0; n < cnt; ++n) {  // row by row: no division in the copy loop
            const __half* src = p.x16 + (size_t)p.pair_token[start + grp * kPreGuGroup + n] * H;
            for (int c = tid * 8; c < H; c += kPreGuThreads * 8)
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(rows_s + n * H + c)), "l"(src + c) : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncthreads();
        // warp -> (position n, stages st0, st0 + W, ...): everything that depends on the position alone is set up once.
        // A warp takes a whole 256-column stage: its two half-warps each transform one 128-block, eight values per lane
        constexpr int W = kPreGuThreads / 32 / kPreGuGroup;
        const int n = warp % kPreGuGroup;
        if (n < cnt) {
            const int pos = grp * kPreGuGroup + n, pair = start + pos;
            const int half = lane >> 4, jl = lane & 15;
            const __half* row = rows_s + n * H + half * 128 + jl * 8;
            const bool plain = e >= L.n_experts;  // shared expert: plain weights, identity keys
            const uint16_t* cin = L.gu_cin + (size_t)(plain ? 0 : e) * H + half * 128 + jl * 8;
            const uint32_t* cs2 = L.gu_cs2 + (size_t)(plain ? 0 : e) * (H / 32) + half * 4 + (jl >> 2);
            uint8_t* img0 = p.bq_gu + (size_t)item * (H / 256) * kWideStageBytes;
            if (warp < kPreGuGroup && lane == 0) p.pscale_gu[pair] = p.tok_scale[p.pair_token[pair]];
            for (int st = warp / kPreGuGroup; st < H / 256; st += W) {
                float v[8];
                if (plain) {
                    const uint4 raw = *reinterpret_cast<const uint4*>(row + st * 256);
                    const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[i]));
                        v[2 * i] = f.x;
                        v[2 * i + 1] = f.y;
                    }
                } else {
                    const uint4 ce = *reinterpret_cast<const uint4*>(cin + st * 256);
                    const uint32_t ent[8] = {ce.x & 0xffffu, ce.x >> 16, ce.y & 0xffffu, ce.y >> 16,
                                             ce.z & 0xffffu, ce.z >> 16, ce.w & 0xffffu, ce.w >> 16};
                    const __half* base = rows_s + n * H;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float xv = __half2float(base[ent[i] & 0x7fffu]);
                        v[i] = (ent[i] >> 15) ? -xv : xv;
                    }
                    fwht128_half(v, lane);
                    const uint32_t sw = cs2[st * 8] >> ((jl & 3) * 8);
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        if ((sw >> i) & 1u) v[i] = -v[i];
                }
                quantize_stage_fp4x3<kWideRows, kPairsPerWideItem>(v, lane, img0 + (size_t)st * kWideStageBytes, pos);
            }
        }
    }
}

int launch_pre_gu(const chronos_layer_t& L, const void* x, int x_dtype, const Plan& p, int fp4, int many_pairs,
                  cudaStream_t st) {
    if (fp4 == 2) {
        const int sms = device_sm_count();
        const size_t smem = (size_t)kPreGuGroup * L.hidden * 2;
        if (int rc = ensure_dynamic_smem(reinterpret_cast<const void*>(pre_gu_wide_kernel), smem, "pre_gu_wide")) return rc;
        const long most = (long)p.max_gitems * (kPairsPerWideItem / kPreGuGroup);
        const long resident = (long)sms * (smem * 4 <= 200 * 1024 ? 4 : (smem * 2 <= 200 * 1024 ? 2 : 1));
        pre_gu_wide_kernel<<<(unsigned)(most < resident ? most : resident), kPreGuThreads, smem, st>>>(L, p);
        return check_launch("pre_gu_wide");
    }
    const long xf = fp4 ? (long)p.max_items * kPairsPerItem * (L.hidden / 128) : (long)p.max_pairs * (L.hidden / 128);
    // few pairs per expert: healer warps ride along in the same launch, one per (pair, rank row); many pairs per expert:
    // a second launch whose blocks share healer rows through L1
    const long warps = xf + (many_pairs ? 0 : (long)p.max_pairs * L.rank);
    pre_gu_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(L, x, x_dtype, p, fp4);
    if (int rc = check_launch("pre_gu")) return rc;
    if (many_pairs != 1) return CHRONOS_OK;  // 2: the caller runs the tensor-core healer kernel instead
    healer_in_tile_kernel<<<(unsigned)(((p.max_pairs + 7) / 8) * (L.rank / 8)), 256, 0, st>>>(L, x, x_dtype, p);
    return check_launch("healer_in_tile");
}

// ---------------------------------------------------------------------------------------------------------------
// Between the passes, part A: SwiGLU outputs in natural order. One warp per (sorted pair, 128 outputs):
// act[i] = silu(z_gu[i]) * z_gu[I + i] with z_gu[row] = beta * r_s1[row] * z1[r_inv[row]] + U_gu[row, :] . hmid;
// also the pair's partial sum of squares of the block and the partial down-healer input V_down . act of the block.
// ---------------------------------------------------------------------------------------------------------------
template <int R16>  // healer rank / 16: compile-time so that every 16-byte healer load of a row can be issued up front
__global__ void __launch_bounds__(256) mid_act_kernel(chronos_layer_t L, Plan p) {
    __shared__ float hs[8][kMaxRank];
    __shared__ float act_s[8][128];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int n_pairs = p.counters[1];
    const int I = L.inter, E = L.n_experts;
    constexpr int r = R16 * 16;
    const int nblk = I / 128;
    // a block = 8 consecutive sorted pairs x one 128-output block: pairs of one expert sit next to each other, so the
    // warps of a block mostly read the same healer rows (L1 hits) when an expert has many pairs
    const int pair = (int)(blockIdx.x / nblk) * 8 + wib, blk = (int)(blockIdx.x % nblk);
    if (pair >= n_pairs) return;
    const int e = p.pair_expert[pair];
    const float* z1 = p.z1 + (size_t)pair * 2 * I;
    const int i0 = blk * 128 + lane * 4;
    float a[4];
    if (e >= E) {  // shared expert: rows in natural order, no healer
        const float4 zg = *reinterpret_cast<const float4*>(z1 + i0);
        const float4 zu = *reinterpret_cast<const float4*>(z1 + I + i0);
        a[0] = silu_f32(zg.x) * zu.x; a[1] = silu_f32(zg.y) * zu.y;
        a[2] = silu_f32(zg.z) * zu.z; a[3] = silu_f32(zg.w) * zu.w;
    } else {
        for (int c = lane; c < r; c += 32) hs[wib][c] = p.hmid[(size_t)pair * r + c];
        __syncwarp();
        const float beta = L.gu_beta[e];
        const uint16_t* rout = L.gu_rout + (size_t)e * 2 * I;
        const uint8_t* ug = L.u_gu + (size_t)e * 2 * I * r;
        float zz[2][4];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const uint2 ro2 = *reinterpret_cast<const uint2*>(rout + half * I + i0);
            const uint32_t ro[4] = {ro2.x & 0xffffu, ro2.x >> 16, ro2.y & 0xffffu, ro2.y >> 16};
            float zb[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float z = z1[ro[q] & 0x7fffu];
                zb[q] = (ro[q] >> 15) ? -z : z;
            }
            const uint4* urow = reinterpret_cast<const uint4*>(ug + (size_t)(half * I + i0) * r);
            uint4 uall[4 * R16];  // rows i0..i0+3 are contiguous: 4 * r bytes
#pragma unroll
            for (int w = 0; w < 4 * R16; ++w) uall[w] = urow[w];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                float heal = 0.0f;
#pragma unroll
                for (int c16 = 0; c16 < R16; ++c16) {
                    const uint4 u = uall[q * R16 + c16];
                    const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                    for (int w4 = 0; w4 < 4; ++w4) {
                        const float2 lo = e4m3x2_to_f32((uint16_t)(uw[w4] & 0xffffu));
                        const float2 hi = e4m3x2_to_f32((uint16_t)(uw[w4] >> 16));
                        const float* hp = &hs[wib][c16 * 16 + w4 * 4];
                        heal = fmaf(lo.x, hp[0], heal);
                        heal = fmaf(lo.y, hp[1], heal);
                        heal = fmaf(hi.x, hp[2], heal);
                        heal = fmaf(hi.y, hp[3], heal);
                    }
                }
                zz[half][q] = fmaf(beta, zb[q], heal);
                if (p.tail_gu) zz[half][q] += p.tail_gu[(size_t)pair * 2 * I + half * I + i0 + q];
            }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) a[q] = silu_f32(zz[0][q]) * zz[1][q];
    }
    *reinterpret_cast<float4*>(p.act + (size_t)pair * I + i0) = make_float4(a[0], a[1], a[2], a[3]);
    float ss = a[0] * a[0] + a[1] * a[1] + a[2] * a[2] + a[3] * a[3];
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) p.act_ss[(size_t)pair * nblk + blk] = ss;
    if (e >= E) return;
    // partial down-healer input: hpart[pair, blk, c] = sum_{i in block} V_down^T[e, i, c] * act[i].
    // A row of V_down^T is r bytes = r/16 chunks of 16; lane = (row selector, chunk): 32/(r/16) rows per step.
    *reinterpret_cast<float4*>(&act_s[wib][lane * 4]) = make_float4(a[0], a[1], a[2], a[3]);
    __syncwarp();
    const uint8_t* vt = L.v_dn_t + ((size_t)e * I + blk * 128) * r;
    constexpr int cpr = R16, rpi = 32 / cpr;
    const int rsel = lane / cpr, chunk = lane % cpr;
    float hacc[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) hacc[c] = 0.0f;
#pragma unroll 8
    for (int j0 = 0; j0 < 128; j0 += rpi) {
        const int jj = j0 + rsel;
        const uint4 w = *reinterpret_cast<const uint4*>(vt + (size_t)jj * r + chunk * 16);
        const float av = act_s[wib][jj];
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float2 lo = e4m3x2_to_f32((uint16_t)(ww[q] & 0xffffu)), hi = e4m3x2_to_f32((uint16_t)(ww[q] >> 16));
            hacc[q * 4 + 0] = fmaf(lo.x, av, hacc[q * 4 + 0]);
            hacc[q * 4 + 1] = fmaf(lo.y, av, hacc[q * 4 + 1]);
            hacc[q * 4 + 2] = fmaf(hi.x, av, hacc[q * 4 + 2]);
            hacc[q * 4 + 3] = fmaf(hi.y, av, hacc[q * 4 + 3]);
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

// Part B: down-input transform of the SwiGLU outputs, fp16 rows (one warp per (pair, block)) or FP4 images
// (one warp per (work item, position, block); the pair's scale comes from the partial sums of squares of part A).
__global__ void __launch_bounds__(256) mid_xform_kernel(chronos_layer_t L, Plan p, int fp4) {
    const int lane = threadIdx.x & 31;
    const long gw = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int I = L.inter, nblk = I / 128;
    float v[4];
    if (!fp4) {
        const int pair = (int)(gw / nblk), blk = (int)(gw % nblk);
        if (pair >= p.counters[1]) return;
        float ss = 0.0f;
        for (int b = 0; b < nblk; ++b) ss += p.act_ss[(size_t)pair * nblk + b];
        const float g = pow2_scale(ss, I);
        transform_dn_block(L, p.act + (size_t)pair * I, p.pair_expert[pair], blk, lane, v);
        const float gi = 1.0f / g;
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] *= gi;
        if (blk == 0 && lane == 0) p.pscale_dn[pair] = g;
        store_half4(p.ac + (size_t)pair * I + blk * 128 + lane * 4, v);
        return;
    }
    const int blk = (int)(gw % nblk);
    const int ip = (int)(gw / nblk), item = ip / kPairsPerItem, pos = ip % kPairsPerItem;
    if (item >= p.counters[0] || pos >= p.item_cnt[item]) return;  // absent pairs: rows left unwritten (see pre_gu_kernel)
    {
        const int pair = p.item_start[item] + pos;
        float ss = 0.0f;
        for (int b = 0; b < nblk; ++b) ss += p.act_ss[(size_t)pair * nblk + b];  // fixed order: same scale in every warp
        const float g = pow2_scale(ss, I);
        transform_dn_block(L, p.act + (size_t)pair * I, p.pair_expert[pair], blk, lane, v);
        const float gi = 1.0f / g;
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] *= gi;
        if (blk == 0 && lane == 0) p.pscale_dn[pair] = g;
    }
    uint8_t* img = p.bq_dn + ((size_t)item * (I / 256) + blk / 2) * 6144;
    quantize_block_fp4x3<32, 8>(v, lane, img, blk & 1, pos);
}

int launch_mid(const chronos_layer_t& L, const Plan& p, int fp4, cudaStream_t st) {
    const int nblk = L.inter / 128;
    long warps = (long)p.max_pairs * nblk;
    const unsigned grid_a = (unsigned)(((p.max_pairs + 7) / 8) * nblk);
    switch (L.rank / 16) {
        case 1: mid_act_kernel<1><<<grid_a, 256, 0, st>>>(L, p); break;
        case 2: mid_act_kernel<2><<<grid_a, 256, 0, st>>>(L, p); break;
        case 4: mid_act_kernel<4><<<grid_a, 256, 0, st>>>(L, p); break;
        default: mid_act_kernel<8><<<grid_a, 256, 0, st>>>(L, p); break;
    }
    if (int rc = check_launch("mid_act")) return rc;
    if (fp4) warps = (long)p.max_items * kPairsPerItem * nblk;
    mid_xform_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(L, p, fp4);
    return check_launch("mid_xform");
}

// ---------------------------------------------------------------------------------------------------------------
// Combine: y[t, i] = sum_j gate[t, j] * (beta_d * r_s1[i] * y1[p_j, r_inv[i]] + U_down[e_j, i, :] . hd[p_j, :])
//                    (+ shared expert row), summed over j = 0..top_k-1 in that order.
// One block per (token, 128 output rows): warp w evaluates routing entries j = w, w+8, ...; lane l owns rows 4l..4l+3;
// the per-entry terms meet in shared memory and are added in index order (deterministic).
// ---------------------------------------------------------------------------------------------------------------
template <int R16>
__global__ void __launch_bounds__(256) combine_kernel(chronos_layer_t L, Plan p, const float* __restrict__ gates,
                                                      int with_shared, void* __restrict__ y, int y_dtype) {
    __shared__ float hd[8][kMaxRank];
    __shared__ __align__(16) float terms[kMaxTopK][128];
    const int t = blockIdx.x, rb = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int H = L.hidden, I = L.inter, E = L.n_experts, k = L.top_k;
    constexpr int r = R16 * 16;
    const int nblk = I / 128;
    const int row0 = rb * 128 + lane * 4;
    for (int j = warp; j < k; j += 8) {
        const int pos = p.pos_of[t * k + j];
        float out[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (pos >= 0) {
            const int e = p.pair_expert[pos];
            // the healer rows of this lane's 4 outputs do not depend on anything computed here: request them first
            const uint4* urow = reinterpret_cast<const uint4*>(L.u_dn + ((size_t)e * H + row0) * r);
            uint4 uall[4 * R16];
#pragma unroll
            for (int w = 0; w < 4 * R16; ++w) uall[w] = urow[w];
            for (int c = lane; c < r; c += 32) {
                float s = 0.0f;
#pragma unroll 4
                for (int b = 0; b < nblk; ++b) s += p.hpart[((size_t)pos * nblk + b) * r + c];
                hd[warp][c] = s;
            }
            __syncwarp();
            const float g = gates[t * k + j], beta = L.dn_beta[e];
            const uint2 ro2 = *reinterpret_cast<const uint2*>(L.dn_rout + (size_t)e * H + row0);
            const uint32_t ro[4] = {ro2.x & 0xffffu, ro2.x >> 16, ro2.y & 0xffffu, ro2.y >> 16};
            float yb[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float v = p.y1[(size_t)pos * H + (ro[q] & 0x7fffu)];
                yb[q] = (ro[q] >> 15) ? -v : v;
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                float heal = 0.0f;
#pragma unroll
                for (int c16 = 0; c16 < R16; ++c16) {
                    const uint4 u = uall[q * R16 + c16];
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
                float term = fmaf(beta, yb[q], heal);
                if (p.tail_dn) term += p.tail_dn[(size_t)pos * H + row0 + q];
                out[q] = g * term;
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
        if (with_shared && t >= p.shared_lo && t < p.shared_lo + p.shared_n)
            acc += p.y1[(size_t)(p.offsets[E] + t - p.shared_lo) * H + i];
        if (y_dtype == CHRONOS_DTYPE_BF16)
            reinterpret_cast<__nv_bfloat16*>(y)[(size_t)t * H + i] = __float2bfloat16(acc);
        else
            reinterpret_cast<float*>(y)[(size_t)t * H + i] = acc;
    }
}

// Tensor-regime combine, part 1: yt[pair, i] = beta_d * r_s1[i] * y1[pair, r_inv[i]] + U_down[e, i, :] . hd[pair, :].
// A block = 8 consecutive sorted pairs x 128 output rows (the warps share the healer rows of an expert through L1).
template <int R16>
__global__ void __launch_bounds__(256) down_term_kernel(chronos_layer_t L, Plan p) {
    __shared__ float hd[8][kMaxRank];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int H = L.hidden, I = L.inter, E = L.n_experts;
    constexpr int r = R16 * 16;
    const int nblk = I / 128, nrb = H / 128;
    const int pos = (int)(blockIdx.x / nrb) * 8 + warp, rb = (int)(blockIdx.x % nrb);
    if (pos >= p.counters[1]) return;
    const int e = p.pair_expert[pos];
    const int row0 = rb * 128 + lane * 4;
    float4* dst = reinterpret_cast<float4*>(p.yt + (size_t)pos * H + row0);
    if (e >= E) {  // shared expert: plain rows
        *dst = *reinterpret_cast<const float4*>(p.y1 + (size_t)pos * H + row0);
        return;
    }
    const uint4* urow = reinterpret_cast<const uint4*>(L.u_dn + ((size_t)e * H + row0) * r);
    uint4 uall[4 * R16];
#pragma unroll
    for (int w = 0; w < 4 * R16; ++w) uall[w] = urow[w];
    for (int c = lane; c < r; c += 32) {
        float s = 0.0f;
#pragma unroll 4
        for (int b = 0; b < nblk; ++b) s += p.hpart[((size_t)pos * nblk + b) * r + c];
        hd[warp][c] = s;
    }
    __syncwarp();
    const float beta = L.dn_beta[e];
    const uint2 ro2 = *reinterpret_cast<const uint2*>(L.dn_rout + (size_t)e * H + row0);
    const uint32_t ro[4] = {ro2.x & 0xffffu, ro2.x >> 16, ro2.y & 0xffffu, ro2.y >> 16};
    float out[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float v = p.y1[(size_t)pos * H + (ro[q] & 0x7fffu)];
        const float yb = (ro[q] >> 15) ? -v : v;
        float heal = 0.0f;
#pragma unroll
        for (int c16 = 0; c16 < R16; ++c16) {
            const uint4 u = uall[q * R16 + c16];
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
        out[q] = fmaf(beta, yb, heal);
        if (p.tail_dn) out[q] += p.tail_dn[(size_t)pos * H + row0 + q];
    }
    *dst = make_float4(out[0], out[1], out[2], out[3]);
}

// Part 2: y[t, i] = sum_j gate[t, j] * yt[pos(t, j), i] (+ shared expert row), j in index order.
__global__ void __launch_bounds__(256) combine_sum_kernel(chronos_layer_t L, Plan p, const float* __restrict__ gates,
                                                          int with_shared, void* __restrict__ y, int y_dtype) {
    const int H = L.hidden, k = L.top_k;
    const int t = blockIdx.x, i0 = (blockIdx.y * 256 + threadIdx.x) * 4;
    if (i0 >= H) return;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int j = 0; j < k; ++j) {
        const int pos = p.pos_of[t * k + j];
        if (pos < 0) continue;
        const float g = gates[t * k + j];
        const float4 v = *reinterpret_cast<const float4*>(p.yt + (size_t)pos * H + i0);
        acc[0] = fmaf(g, v.x, acc[0]); acc[1] = fmaf(g, v.y, acc[1]);
        acc[2] = fmaf(g, v.z, acc[2]); acc[3] = fmaf(g, v.w, acc[3]);
    }
    if (with_shared && t >= p.shared_lo && t < p.shared_lo + p.shared_n) {
        const float4 v = *reinterpret_cast<const float4*>(p.yt + (size_t)(p.offsets[L.n_experts] + t - p.shared_lo) * H + i0);
        acc[0] += v.x; acc[1] += v.y; acc[2] += v.z; acc[3] += v.w;
    }
    if (y_dtype == CHRONOS_DTYPE_BF16) {
        __nv_bfloat162 a01 = __floats2bfloat162_rn(acc[0], acc[1]), a23 = __floats2bfloat162_rn(acc[2], acc[3]);
        uint2 o;
        o.x = *reinterpret_cast<uint32_t*>(&a01);
        o.y = *reinterpret_cast<uint32_t*>(&a23);
        *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(y) + (size_t)t * H + i0) = o;
    } else {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(y) + (size_t)t * H + i0) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    }
}

int launch_combine_tiled(const chronos_layer_t& L, const Plan& p, const float* gates, int n_tokens, int with_shared, void* y,
                         int y_dtype, cudaStream_t st) {
    if (n_tokens <= 0) return CHRONOS_OK;
    const unsigned grid = (unsigned)(((p.max_pairs + 7) / 8) * (L.hidden / 128));
    switch (L.rank / 16) {
        case 1: down_term_kernel<1><<<grid, 256, 0, st>>>(L, p); break;
        case 2: down_term_kernel<2><<<grid, 256, 0, st>>>(L, p); break;
        case 4: down_term_kernel<4><<<grid, 256, 0, st>>>(L, p); break;
        default: down_term_kernel<8><<<grid, 256, 0, st>>>(L, p); break;
    }
    if (int rc = check_launch("down_term")) return rc;
    return launch_combine_sum(L, p, gates, n_tokens, with_shared, y, y_dtype, st);
}

int launch_combine_sum(const chronos_layer_t& L, const Plan& p, const float* gates, int n_tokens, int with_shared, void* y,
                       int y_dtype, cudaStream_t st) {
    if (n_tokens <= 0) return CHRONOS_OK;
    dim3 g2((unsigned)n_tokens, (unsigned)((L.hidden / 4 + 255) / 256));
    combine_sum_kernel<<<g2, 256, 0, st>>>(L, p, gates, with_shared && L.shared_inter > 0, y, y_dtype);
    return check_launch("combine_sum");
}

int launch_combine(const chronos_layer_t& L, const Plan& p, const float* gates, int n_tokens, int with_shared, void* y,
                   int y_dtype, cudaStream_t st) {
    if (n_tokens <= 0) return CHRONOS_OK;
    dim3 grid((unsigned)n_tokens, (unsigned)(L.hidden / 128));
    const int ws = with_shared && L.shared_inter > 0;
    switch (L.rank / 16) {
        case 1: combine_kernel<1><<<grid, 256, 0, st>>>(L, p, gates, ws, y, y_dtype); break;
        case 2: combine_kernel<2><<<grid, 256, 0, st>>>(L, p, gates, ws, y, y_dtype); break;
        case 4: combine_kernel<4><<<grid, 256, 0, st>>>(L, p, gates, ws, y, y_dtype); break;
        default: combine_kernel<8><<<grid, 256, 0, st>>>(L, p, gates, ws, y, y_dtype); break;
    }
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
