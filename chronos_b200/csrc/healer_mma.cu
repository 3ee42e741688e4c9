// Healer products and the transforms between the bank passes for batches with many pairs per expert: the rank-r
// factors run on the tensor cores (mma.sync m16n8k16, fp16 operands converted exactly from e4m3, fp32 accumulate),
// because a CUDA-core e4m3 decode per multiply costs more than the multiply.
// Mathematics as in csrc/transform_kernels.cu (ChronosGlm5HolographicExpertGroup.forward_cold_fast,
// chronos_1t/models/glm5_chronos_moe.py:149-195):
//   hmid = V_gu x;  z_gu = beta r_s1 z1[r_inv] + U_gu hmid;  act = silu(z_gu[:I]) z_gu[I:];
//   hd = V_down act;  y_pair = beta_d r_s1 y1[r_inv] + U_down hd.
//
// Contraction index trick shared by all kernels here: a k16 step of the MMA wants lane (g = lane / 4, q = lane % 4) to
// hold A[row g][2q, 2q+1] and A[row g][2q+8, 2q+9]. Any permutation of the contraction index is legal if A and B
// agree, so lane q owns a CONTIGUOUS run of the row (W 32-bit words of e4m3 = 4 W columns starting at 4 W q), and
// step s takes word s of that run: columns 4Wq + 4s + {0,1} for the low pair, + {2,3} for the high pair. Loads are
// then 4W-byte vectors per lane on the e4m3 side and 8-byte fp16 vectors on the activation side.
#include "common.cuh"

namespace chronos {

__device__ __forceinline__ void cp_async16_g2s(void* smem_dst, const void* gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}


// ---------------------------------------------------------------------------------------------------------------
// Healer input factor of a tensor-regime work item (one expert, up to 128 sorted pairs):
//   out[slice][pair, c] = (1 / g_pair) * sum_{k in slice} V[e, c, k] * X[row(pair), k]      c < r, fp32 partial sums
// V e4m3 [E, r, K]; X rows are activations (bf16 / fp32, or the fp16 image already divided by the token scale; row =
// token of the pair) or SwiGLU outputs (fp32, or fp16 already divided by the pair scale; row = pair);
// g_pair is the power-of-two scale the bank pass uses for the same pair (so the fp16 image stays in range); the
// consumer adds the slices in order and multiplies the scale back. One CTA per (work item, slice of K): the kernel is
// a chain of dependent L2 round trips, so more CTAs in flight is what shortens it. Warp w owns rank rows 16 (w % MT) .. +15 and the pairs of
// 8-pair tiles (w / MT), (w / MT) + 8 / MT, ...
// ---------------------------------------------------------------------------------------------------------------
struct HealInArgs {
    const uint8_t* v;           // [E, r, K]
    const void* x; int x_dtype; // rows of K
    const int32_t* row_of_pair; // NULL: row = pair
    const float* pscale;        // [P]
    float* out;                 // [kHealSplit][P, r] partial sums over the slices of K (slices past n_split stay unwritten)
    size_t split_stride;        // P * r
    int n_split;
    const int32_t* gitem_start; const int32_t* gitem_cnt; const int32_t* pair_expert; const int32_t* counters;
    int K, r, n_experts;
};

template <int MT>  // rank / 16
__global__ void __launch_bounds__(256) healer_in_mma_kernel(const HealInArgs a) {
    constexpr int NG = 8 / MT;        // groups of warps along the pairs
    constexpr int NTW = 16 / NG;      // 8-pair tiles per warp
    const int item = blockIdx.x;
    if (item >= a.counters[3]) return;
    const int start = a.gitem_start[item], cnt = a.gitem_cnt[item];
    const int e = a.pair_expert[start];
    if (e >= a.n_experts) return;     // shared expert: no healer
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, q = lane & 3;
    const int mt = warp % MT, ng = warp / MT;
    const int K = a.K, r = a.r;
    const int ntiles = (cnt + 7) >> 3;
    float acc[NTW][4];
    const uint8_t* xrow[NTW];
    float inv[NTW];
#pragma unroll
    for (int i = 0; i < NTW; ++i) {
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
        const int n = (ng + i * NG) * 8 + g;
        const bool valid = n < cnt;
        const int pair = start + (valid ? n : 0);
        const size_t row = a.row_of_pair ? (size_t)a.row_of_pair[pair] : (size_t)pair;
        xrow[i] = reinterpret_cast<const uint8_t*>(a.x) + row * K * (a.x_dtype == CHRONOS_DTYPE_F32 ? 4 : 2);
        inv[i] = valid ? 1.0f / a.pscale[pair] : 0.0f;
    }
    const uint8_t* v0 = a.v + ((size_t)e * r + mt * 16 + g) * K + 16 * q;
    const uint8_t* v1 = v0 + (size_t)8 * K;
    const int k_lo = (int)blockIdx.y * (K / a.n_split), k_hi = k_lo + K / a.n_split;
#pragma unroll 2
    for (int kc = k_lo; kc < k_hi; kc += 64) {
        const uint4 w0 = *reinterpret_cast<const uint4*>(v0 + kc);
        const uint4 w1 = *reinterpret_cast<const uint4*>(v1 + kc);
        const uint32_t r0[4] = {w0.x, w0.y, w0.z, w0.w}, r1[4] = {w1.x, w1.y, w1.z, w1.w};
        uint32_t af[4][4];
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            af[s][0] = e4m3x2_to_f16x2(r0[s] & 0xffffu);
            af[s][1] = e4m3x2_to_f16x2(r1[s] & 0xffffu);
            af[s][2] = e4m3x2_to_f16x2(r0[s] >> 16);
            af[s][3] = e4m3x2_to_f16x2(r1[s] >> 16);
        }
#pragma unroll
        for (int i = 0; i < NTW; ++i) {
            if (ng + i * NG >= ntiles) continue;  // warp-uniform
            uint32_t bf[8];                       // 16 columns kc + 16 q .. + 15 of this lane's pair, as fp16 pairs
            if (a.x_dtype == kDtypeF16Scaled) {   // already fp16 and divided by the pair's scale: no conversion work
                const uint4* src = reinterpret_cast<const uint4*>(xrow[i] + (size_t)(kc + 16 * q) * 2);
                const uint4 u0 = src[0], u1 = src[1];
                bf[0] = u0.x; bf[1] = u0.y; bf[2] = u0.z; bf[3] = u0.w;
                bf[4] = u1.x; bf[5] = u1.y; bf[6] = u1.z; bf[7] = u1.w;
            } else if (a.x_dtype == CHRONOS_DTYPE_BF16) {
                const uint4* src = reinterpret_cast<const uint4*>(xrow[i] + (size_t)(kc + 16 * q) * 2);
                const uint4 u0 = src[0], u1 = src[1];
                const uint32_t uu[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    bf[j] = pack_f16x2_sat(__uint_as_float(uu[j] << 16) * inv[i], __uint_as_float(uu[j] & 0xffff0000u) * inv[i]);
            } else {
                const float4* src = reinterpret_cast<const float4*>(xrow[i] + (size_t)(kc + 16 * q) * 4);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float4 f = src[j];
                    bf[2 * j] = pack_f16x2_sat(f.x * inv[i], f.y * inv[i]);
                    bf[2 * j + 1] = pack_f16x2_sat(f.z * inv[i], f.w * inv[i]);
                }
            }
#pragma unroll
            for (int s = 0; s < 4; ++s) mma_16816(acc[i], af[s][0], af[s][1], af[s][2], af[s][3], bf[2 * s], bf[2 * s + 1]);
        }
    }
#pragma unroll
    for (int i = 0; i < NTW; ++i) {
        if (ng + i * NG >= ntiles) continue;
        const int n0 = (ng + i * NG) * 8 + 2 * q;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + (j & 1), c = mt * 16 + g + (j >> 1) * 8;
            if (n < cnt) a.out[blockIdx.y * a.split_stride + (size_t)(start + n) * r + c] = acc[i][j];
        }
    }
}

// The same product for fp16 rows that are already divided by the pair's scale (the FP4 tensor regime hands both stages
// over in that form), with the operands staged through shared memory by a ring of asynchronous 16-byte copies:
// kRingStages - 1 steps of 64 columns are in flight while one is multiplied, so the kernel no longer waits a full
// L2 round trip per step, every activation row is fetched once per CTA instead of once per rank-row warp, and the loads
// in flight do not cost registers. Fragment ownership as above; a step's tile is X [ROWS pairs][64 fp16] with rows
// padded to 144 bytes and V [r][64 e4m3] unpadded (both conflict-free for the 16-byte fragment reads).
constexpr int kRingStages = 4;
constexpr int kRingXStride = 144;

template <int MT, int ROWS>  // rank / 16; pairs of a work item at most (64 or 128)
__global__ void __launch_bounds__(256) healer_in_ring_kernel(const HealInArgs a) {
    extern __shared__ __align__(16) uint8_t ring[];
    constexpr int r = MT * 16;
    constexpr int NG = 8 / MT, NTW = (ROWS / 8) / NG;
    constexpr int kXBytes = ROWS * kRingXStride, kStage = kXBytes + r * 64;
    constexpr int XJ = ROWS * 8 / 256;                 // 16-byte activation chunks per thread and step
    constexpr int VJ = (r * 4 + 255) / 256;            // healer chunks per thread and step
    const int item = blockIdx.x;
    if (item >= a.counters[3]) return;
    const int start = a.gitem_start[item], cnt = a.gitem_cnt[item];
    const int e = a.pair_expert[start];
    if (e >= a.n_experts) return;     // shared expert: no healer
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, q = lane & 3;
    const int mt = warp % MT, ng = warp / MT;
    const int K = a.K;
    const int ntiles = (cnt + 7) >> 3;
    const int k_lo = (int)blockIdx.y * (K / a.n_split), n_steps = (K / a.n_split) / 64;
    const uint8_t* xsrc[XJ];
    bool xok[XJ];
#pragma unroll
    for (int j = 0; j < XJ; ++j) {
        const int c = tid + 256 * j, row = c >> 3;
        xok[j] = row < cnt;
        const int pair = start + (xok[j] ? row : 0);
        const size_t src_row = a.row_of_pair ? (size_t)a.row_of_pair[pair] : (size_t)pair;
        xsrc[j] = reinterpret_cast<const uint8_t*>(a.x) + (src_row * K + k_lo + (c & 7) * 8) * 2;
    }
    const uint8_t* vsrc = a.v + (size_t)e * r * K + k_lo;
    auto issue = [&](int step) {
        uint8_t* slot = ring + (step % kRingStages) * kStage;
#pragma unroll
        for (int j = 0; j < XJ; ++j) {
            const int c = tid + 256 * j;
            if (xok[j]) cp_async16_g2s(slot + (c >> 3) * kRingXStride + (c & 7) * 16, xsrc[j] + (size_t)step * 128);
        }
#pragma unroll
        for (int j = 0; j < VJ; ++j) {
            const int c = tid + 256 * j;
            if (c < r * 4) cp_async16_g2s(slot + kXBytes + c * 16, vsrc + (size_t)(c >> 2) * K + step * 64 + (c & 3) * 16);
        }
    };
    // rows of absent pairs are never copied: clear them once so that the unused MMA columns stay finite
    for (int i = tid; i < kRingStages * ROWS * (kRingXStride / 16); i += 256) {
        const int stg = i / (ROWS * (kRingXStride / 16)), rem = i % (ROWS * (kRingXStride / 16));
        if (rem / (kRingXStride / 16) >= cnt)
            *reinterpret_cast<uint4*>(ring + stg * kStage + rem * 16) = make_uint4(0u, 0u, 0u, 0u);
    }
    float acc[NTW][4];
#pragma unroll
    for (int i = 0; i < NTW; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
#pragma unroll
    for (int s0 = 0; s0 < kRingStages - 1; ++s0) {
        if (s0 < n_steps) issue(s0);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    for (int step = 0; step < n_steps; ++step) {
        asm volatile("cp.async.wait_group %0;" ::"n"(kRingStages - 2) : "memory");
        __syncthreads();  // the step's tile has landed for every thread; the slot refilled next was read one step ago
        if (step + kRingStages - 1 < n_steps) issue(step + kRingStages - 1);
        asm volatile("cp.async.commit_group;" ::: "memory");
        const uint8_t* slot = ring + (step % kRingStages) * kStage;
        const uint4 w0 = *reinterpret_cast<const uint4*>(slot + kXBytes + (mt * 16 + g) * 64 + 16 * q);
        const uint4 w1 = *reinterpret_cast<const uint4*>(slot + kXBytes + (mt * 16 + g + 8) * 64 + 16 * q);
        const uint32_t r0[4] = {w0.x, w0.y, w0.z, w0.w}, r1[4] = {w1.x, w1.y, w1.z, w1.w};
        uint32_t af[4][4];
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            af[s][0] = e4m3x2_to_f16x2(r0[s] & 0xffffu);
            af[s][1] = e4m3x2_to_f16x2(r1[s] & 0xffffu);
            af[s][2] = e4m3x2_to_f16x2(r0[s] >> 16);
            af[s][3] = e4m3x2_to_f16x2(r1[s] >> 16);
        }
#pragma unroll
        for (int i = 0; i < NTW; ++i) {
            if (ng + i * NG >= ntiles) continue;  // warp-uniform
            const uint4* src = reinterpret_cast<const uint4*>(slot + ((ng + i * NG) * 8 + g) * kRingXStride + 32 * q);
            const uint4 u0 = src[0], u1 = src[1];
            const uint32_t bf[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
            for (int s = 0; s < 4; ++s) mma_16816(acc[i], af[s][0], af[s][1], af[s][2], af[s][3], bf[2 * s], bf[2 * s + 1]);
        }
    }
#pragma unroll
    for (int i = 0; i < NTW; ++i) {
        if (ng + i * NG >= ntiles) continue;
        const int n0 = (ng + i * NG) * 8 + 2 * q;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + (j & 1), c = mt * 16 + g + (j >> 1) * 8;
            if (n < cnt) a.out[blockIdx.y * a.split_stride + (size_t)(start + n) * r + c] = acc[i][j];
        }
    }
}

template <int MT, int ROWS>
static int launch_healer_ring(const HealInArgs& a, dim3 grid, cudaStream_t st) {
    const size_t smem = (size_t)kRingStages * (ROWS * kRingXStride + MT * 16 * 64);
    if (int rc = ensure_dynamic_smem(reinterpret_cast<const void*>(healer_in_ring_kernel<MT, ROWS>), smem, "healer_in_ring")) return rc;
    healer_in_ring_kernel<MT, ROWS><<<grid, 256, smem, st>>>(a);
    return check_launch("healer_in_ring");
}

// Fused healer of the FP4 tensor regime: the healer input factors of a work item (the sum, in slice order, of the
// partial sums above; still divided by the pair scale) times the layer's power-of-two tile scale, as the K-major fp16
// operand tile the bank pass multiplies with the healer tiles: half (c, pos) at (c / 8) * 512 + pos * 8 + c % 8.
// Positions past the item's count are zero. One CTA per work item; the shared expert has no healer.
__global__ void __launch_bounds__(256) heal_image_kernel(const float* __restrict__ hsplit, size_t split_stride, int n_split, int r,
                                                         const float* __restrict__ tile_scale, const int32_t* __restrict__ gitem_start,
                                                         const int32_t* __restrict__ gitem_cnt, const int32_t* __restrict__ pair_expert,
                                                         const int32_t* __restrict__ counters, int n_experts, __half* __restrict__ himg) {
    const int item = blockIdx.x;
    if (item >= counters[3]) return;
    const int start = gitem_start[item], cnt = gitem_cnt[item];
    if (pair_expert[start] >= n_experts) return;
    const float k = *tile_scale;
    __half* img = himg + (size_t)item * kPairsPerWideItem * r;
    for (int idx = threadIdx.x * 4; idx < kPairsPerWideItem * r; idx += 256 * 4) {
        const int pos = idx / r, c = idx % r;  // 4 consecutive rank columns of one position
        float4 acc4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (pos < cnt) {
            float4 part[kHealSplit];
#pragma unroll
            for (int ks = 0; ks < kHealSplit; ++ks) {
                part[ks] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (ks < n_split) part[ks] = *reinterpret_cast<const float4*>(hsplit + ks * split_stride + (size_t)(start + pos) * r + c);
            }
            acc4 = part[0];
#pragma unroll
            for (int ks = 1; ks < kHealSplit; ++ks) {
                acc4.x += part[ks].x; acc4.y += part[ks].y; acc4.z += part[ks].z; acc4.w += part[ks].w;
            }
        }
        const float h4[4] = {acc4.x * k, acc4.y * k, acc4.z * k, acc4.w * k};
        store_half4(img + (c >> 3) * (kPairsPerWideItem * 8) + pos * 8 + (c & 7), h4);
    }
}

int launch_heal_image(const chronos_layer_t& L, int stage, const Plan& p, cudaStream_t st) {
    const size_t sstride = (size_t)p.max_pairs * L.rank;
    const int kdim = stage == 0 ? L.hidden : L.inter;
    const int n_split = kdim % (64 * kHealSplit) == 0 ? kHealSplit : (kdim % 128 == 0 ? 2 : 1);
    heal_image_kernel<<<(unsigned)p.max_gitems, 256, 0, st>>>(p.hsplit + (size_t)stage * kHealSplit * sstride, sstride, n_split, L.rank,
                                                              L.ut_scale + stage, p.gitem_start, p.gitem_cnt, p.pair_expert, p.counters,
                                                              L.n_experts, p.himg);
    return check_launch("heal_image");
}

int launch_healer_in_mma(const chronos_layer_t& L, int stage, const void* x, int x_dtype, const Plan& p, cudaStream_t st) {
    HealInArgs a{};
    a.v = stage == 0 ? L.v_gu : L.v_dn;
    a.x = x;             // stage 0: token rows; stage 1: SwiGLU outputs per pair (fp32 p.act, or fp16 rows in p.ac)
    a.x_dtype = x_dtype;
    a.row_of_pair = stage == 0 ? p.pair_token : nullptr;
    a.pscale = stage == 0 ? p.pscale_gu : p.pscale_dn;
    a.split_stride = (size_t)p.max_pairs * L.rank;
    a.out = p.hsplit + (size_t)stage * kHealSplit * a.split_stride;
    const int kdim = stage == 0 ? L.hidden : L.inter;
    a.n_split = kdim % (64 * kHealSplit) == 0 ? kHealSplit : (kdim % 128 == 0 ? 2 : 1);
    a.gitem_start = p.gitem_start;
    a.gitem_cnt = p.gitem_cnt;
    a.pair_expert = p.pair_expert;
    a.counters = p.counters;
    a.K = stage == 0 ? L.hidden : L.inter;
    a.r = L.rank;
    a.n_experts = L.n_experts;
    const dim3 grid((unsigned)p.max_gitems, (unsigned)a.n_split);
    if (x_dtype == kDtypeF16Scaled && (a.K / a.n_split) % 64 == 0) {
        const bool small = p.gitem_pairs <= 64;
        switch (L.rank / 16) {
            case 1: return small ? launch_healer_ring<1, 64>(a, grid, st) : launch_healer_ring<1, 128>(a, grid, st);
            case 2: return small ? launch_healer_ring<2, 64>(a, grid, st) : launch_healer_ring<2, 128>(a, grid, st);
            case 4: return small ? launch_healer_ring<4, 64>(a, grid, st) : launch_healer_ring<4, 128>(a, grid, st);
            default: return small ? launch_healer_ring<8, 64>(a, grid, st) : launch_healer_ring<8, 128>(a, grid, st);
        }
    }
    switch (L.rank / 16) {
        case 1: healer_in_mma_kernel<1><<<grid, 256, 0, st>>>(a); break;
        case 2: healer_in_mma_kernel<2><<<grid, 256, 0, st>>>(a); break;
        case 4: healer_in_mma_kernel<4><<<grid, 256, 0, st>>>(a); break;
        default: healer_in_mma_kernel<8><<<grid, 256, 0, st>>>(a); break;
    }
    return check_launch("healer_in_mma");
}

// ---------------------------------------------------------------------------------------------------------------
// Output side of a bank pass for a group of kGroupPairs sorted pairs of one expert (a sub-range of a tensor-regime work
// item). The pairs' bank-pass outputs (permuted row order, fp32) are staged in shared memory with asynchronous 16-byte
// copies, so the inverse-permutation gather runs in shared memory. Then, 16 output rows at a time per warp,
//   D[row, pair] = U[e, row, :] . h[pair, :]      (tensor cores; U rows converted e4m3 -> fp16 in registers; the MMA's
//                                                  8 pair columns are half used - the healer FLOPs are negligible)
//   z[row, pair] = beta * sign * vec[pair][r_inv[row]] + g_pair * D[row, pair].
// MODE 0 (gate_up): rows come in (gate, up) couples; act = silu(z_gate) * z_up is kept in shared memory, then per
//   pair the power-of-two scale of the down pass, the natural-order copy for the down healer, and the down-input
//   transform (gather + sign, FWHT128, sign) written as fp16 rows or as an FP4 image.
// MODE 1 (down): z is the pair's layer-output term, stored in natural row order for the gate-weighted sum.
// Small groups keep the shared-memory footprint at a third of an SM, so three CTAs overlap each other's latencies.
// ---------------------------------------------------------------------------------------------------------------
constexpr int kOutThreads = 512;
constexpr int kGroupsPerItem = 128 / kGroupPairs;

template <int MODE, int R16, bool WIDE>  // WIDE: the down input goes out as an FP4 tensor-regime image, not as fp16 rows
__global__ void __launch_bounds__(kOutThreads, 1) pair_group_out_kernel(chronos_layer_t L, Plan p) {
    extern __shared__ __align__(16) float smem_f[];
    __shared__ __align__(16) __half hsm[kGroupPairs][kMaxRank];
    constexpr int PG = kGroupPairs, NW = kOutThreads / 32;
    constexpr int r = R16 * 16;
    const int H = L.hidden, I = L.inter;
    const int VL = MODE == 0 ? 2 * I : H;      // length of a staged vector
    const int NR = MODE == 0 ? I : H;          // output rows (gate/up couples count once)
    float* vec = smem_f;                       // [PG][VL]
    float* acts = smem_f + (size_t)PG * VL;    // MODE 0: [PG][I]
    const float* src = MODE == 0 ? p.z1 : p.y1;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, q = lane & 3;
    // grid-stride over (group, work item), work item fastest so that neighbouring CTAs get comparable work; the bound
    // comes from the device-side item count, so a launch sized for the worst case costs nothing extra
    const int n_items = p.counters[3];
    for (int w = blockIdx.x; w < n_items * kGroupsPerItem; w += gridDim.x) {
        const int sub = w / n_items, item = w % n_items;
        const int cnt = min(PG, p.gitem_cnt[item] - sub * PG);
        if (cnt <= 0) continue;
        __syncthreads();  // shared memory of the previous iteration is no longer read
        const int p0 = p.gitem_start[item] + sub * PG;
        const int e = p.pair_expert[p0];
        if (e >= L.n_experts) {  // shared expert: plain rows, no healer, identity keys
            if constexpr (MODE == 1) {
                for (int i = tid * 4; i < cnt * H; i += kOutThreads * 4)
                    *reinterpret_cast<float4*>(p.yt + (size_t)p0 * H + i) = *reinterpret_cast<const float4*>(src + (size_t)p0 * H + i);
                continue;
            } else {
                for (int n = 0; n < cnt; ++n)
                    for (int i = tid; i < I; i += kOutThreads) {
                        const float zg = src[(size_t)(p0 + n) * 2 * I + i], zu = src[(size_t)(p0 + n) * 2 * I + I + i];
                        acts[n * I + i] = silu_f32(zg) * zu;
                    }
            }
        } else {
            for (int i = tid * 4; i < PG * VL; i += kOutThreads * 4) {
                if (i / VL < cnt) cp_async16_g2s(vec + i, src + (size_t)p0 * VL + i);
                else *reinterpret_cast<float4*>(vec + i) = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
            // healer input factors of the group: the sum, in slice order, of the healer-input kernel's partial sums, as
            // fp16 in shared memory (rows of absent pairs are zero)
            const size_t sstride = (size_t)p.max_pairs * r;
            const float* hs = p.hsplit + (size_t)MODE * kHealSplit * sstride;
            const int kdim = MODE == 0 ? H : I;
            const int n_split = kdim % (64 * kHealSplit) == 0 ? kHealSplit : (kdim % 128 == 0 ? 2 : 1);
            if (tid < PG * (r / 4)) {
                const int n = tid / (r / 4), c4 = (tid % (r / 4)) * 4;
                float4 part[kHealSplit];
#pragma unroll
                for (int ks = 0; ks < kHealSplit; ++ks) {  // all slices requested before any is added
                    part[ks] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    if (n < cnt && ks < n_split) part[ks] = *reinterpret_cast<const float4*>(hs + ks * sstride + (size_t)(p0 + n) * r + c4);
                }
                float4 acc4 = part[0];
#pragma unroll
                for (int ks = 1; ks < kHealSplit; ++ks) {
                    acc4.x += part[ks].x; acc4.y += part[ks].y; acc4.z += part[ks].z; acc4.w += part[ks].w;
                }
                const float h4[4] = {acc4.x, acc4.y, acc4.z, acc4.w};
                store_half4(&hsm[n][c4], h4);
            }
            const float* psc = MODE == 0 ? p.pscale_gu : p.pscale_dn;
            const float gs0 = 2 * q < cnt ? psc[p0 + 2 * q] : 0.0f, gs1 = 2 * q + 1 < cnt ? psc[p0 + 2 * q + 1] : 0.0f;
            const float beta = (MODE == 0 ? L.gu_beta : L.dn_beta)[e];
            const uint16_t* rout = (MODE == 0 ? L.gu_rout : L.dn_rout) + (size_t)e * VL;
            const uint8_t* U = (MODE == 0 ? L.u_gu : L.u_dn) + (size_t)e * VL * r;
            asm volatile("cp.async.wait_all;" ::: "memory");
            __syncthreads();
            // B fragments: h[pair g][4 R16 q + 4 s .. + 3] as two fp16 pairs per step
            uint32_t bf[R16][2];
#pragma unroll
            for (int s = 0; s < R16; ++s) {
                const uint2 v = *reinterpret_cast<const uint2*>(&hsm[g][4 * R16 * q + 4 * s]);
                bf[s][0] = v.x;
                bf[s][1] = v.y;
            }
            // software pipeline over the 16-row tiles of this warp: the healer rows and permutation entries of the next
            // tile are requested before the current tile is multiplied (each request is a full L2 round trip)
            constexpr int NH = MODE == 0 ? 2 : 1;
            auto fetch = [&](int jt, uint32_t (&wl)[NH][R16], uint32_t (&wh)[NH][R16], uint32_t (&rl)[NH], uint32_t (&rh)[NH]) {
#pragma unroll
                for (int half = 0; half < NH; ++half) {
                    const int row_lo = half * I + jt * 16 + g, row_hi = row_lo + 8;
                    const uint32_t* u_lo = reinterpret_cast<const uint32_t*>(U + (size_t)row_lo * r + 4 * R16 * q);
                    const uint32_t* u_hi = reinterpret_cast<const uint32_t*>(U + (size_t)row_hi * r + 4 * R16 * q);
                    if constexpr (R16 % 4 == 0) {
#pragma unroll
                        for (int s = 0; s < R16; s += 4) {
                            const uint4 a4 = *reinterpret_cast<const uint4*>(u_lo + s), b4 = *reinterpret_cast<const uint4*>(u_hi + s);
                            wl[half][s] = a4.x; wl[half][s + 1] = a4.y; wl[half][s + 2] = a4.z; wl[half][s + 3] = a4.w;
                            wh[half][s] = b4.x; wh[half][s + 1] = b4.y; wh[half][s + 2] = b4.z; wh[half][s + 3] = b4.w;
                        }
                    } else {
#pragma unroll
                        for (int s = 0; s < R16; ++s) { wl[half][s] = u_lo[s]; wh[half][s] = u_hi[s]; }
                    }
                    rl[half] = rout[row_lo];
                    rh[half] = rout[row_hi];
                }
            };
            // DEPTH tiles are in flight per warp (register buffers, rotated by unrolling): with one tile in flight an
            // iteration lasted a full L2 round trip whatever it computed
            auto compute = [&](int jt, const uint32_t (&wl)[NH][R16], const uint32_t (&wh)[NH][R16], const uint32_t (&rl)[NH],
                               const uint32_t (&rh)[NH]) {
                const int row_lo = jt * 16 + g, row_hi = row_lo + 8;
                float zz[NH][4];
#pragma unroll
                for (int half = 0; half < NH; ++half) {
                    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                    for (int s = 0; s < R16; ++s)
                        mma_16816(d, e4m3x2_to_f16x2(wl[half][s] & 0xffffu), e4m3x2_to_f16x2(wh[half][s] & 0xffffu),
                                  e4m3x2_to_f16x2(wl[half][s] >> 16), e4m3x2_to_f16x2(wh[half][s] >> 16), bf[s][0], bf[s][1]);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {  // d[j]: row (j < 2 ? lo : hi), pair 2q + (j & 1)
                        const uint32_t ro = j < 2 ? rl[half] : rh[half];
                        const int n = 2 * q + (j & 1);
                        float v = 0.0f;
                        if (n < PG) v = vec[(size_t)n * VL + (ro & 0x7fffu)];
                        zz[half][j] = fmaf(beta, (ro >> 15) ? -v : v, ((j & 1) ? gs1 : gs0) * d[j]);
                        const float* tl = MODE == 0 ? p.tail_gu : p.tail_dn;  // tail-lattice term, natural row order
                        if (tl != nullptr && n < cnt) zz[half][j] += tl[(size_t)(p0 + n) * VL + half * I + (j < 2 ? row_lo : row_hi)];
                    }
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int n = 2 * q + (j & 1), row = j < 2 ? row_lo : row_hi;
                    if (MODE == 0) {
                        if (n < PG) acts[n * I + row] = silu_f32(zz[0][j]) * zz[NH - 1][j];
                    } else if (n < cnt) {
                        p.yt[(size_t)(p0 + n) * H + row] = zz[0][j];
                    }
                }
            };
            constexpr int DEPTH = MODE == 0 ? 2 : 3;
            const int NT = NR / 16;
            uint32_t w_lo[DEPTH][NH][R16], w_hi[DEPTH][NH][R16], ro_lo[DEPTH][NH], ro_hi[DEPTH][NH];
#pragma unroll
            for (int dd = 0; dd < DEPTH; ++dd)
                if (warp + dd * NW < NT) fetch(warp + dd * NW, w_lo[dd], w_hi[dd], ro_lo[dd], ro_hi[dd]);
            for (int jt0 = warp; jt0 < NT; jt0 += DEPTH * NW) {
#pragma unroll
                for (int dd = 0; dd < DEPTH; ++dd) {
                    const int jt = jt0 + dd * NW;
                    if (jt < NT) {  // warp-uniform
                        compute(jt, w_lo[dd], w_hi[dd], ro_lo[dd], ro_hi[dd]);
                        if (jt + DEPTH * NW < NT) fetch(jt + DEPTH * NW, w_lo[dd], w_hi[dd], ro_lo[dd], ro_hi[dd]);
                    }
                }
            }
        }
        if (MODE == 1) continue;
        __syncthreads();
        // per pair: scale of the down pass, natural-order copy, down-input transform; warp w serves pair w % PG and the
        // 128-blocks w / PG, w / PG + NW / PG, ...
        for (int n = warp % PG; n < cnt; n += PG) {
            const float* an = acts + (size_t)n * I;
            float ss = 0.0f;
            for (int i = lane * 4; i < I; i += 128) {
                const float4 v = *reinterpret_cast<const float4*>(an + i);
                ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
            }
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
            const float gsc = pow2_scale(ss, I), gi = 1.0f / gsc;
            const int pair = p0 + n, wsel = warp / PG;
            if (wsel == 0 && lane == 0) p.pscale_dn[pair] = gsc;
            for (int blk = wsel; blk < I / 128; blk += NW / PG) {
                {   // natural-order copy for the down healer: fp16 / pair scale (FP4 regime; p.ac is free there) or fp32
                    const float4 a4 = *reinterpret_cast<const float4*>(an + blk * 128 + lane * 4);
                    if (WIDE) {
                        const float s4[4] = {a4.x * gi, a4.y * gi, a4.z * gi, a4.w * gi};
                        store_half4(p.ac + (size_t)pair * I + blk * 128 + lane * 4, s4);
                    } else {
                        *reinterpret_cast<float4*>(p.act + (size_t)pair * I + blk * 128 + lane * 4) = a4;
                    }
                }
                float v[4];
                transform_dn_block(L, an, e, blk, lane, v);
#pragma unroll
                for (int i = 0; i < 4; ++i) v[i] *= gi;
                if (WIDE) {
                    uint8_t* img = p.bq_dn + ((size_t)item * (I / 256) + blk / 2) * kWideStageBytes;
                    quantize_block_fp4x3<kWideRows, kPairsPerWideItem>(v, lane, img, blk & 1, sub * PG + n);
                } else {
                    store_half4(p.ac + (size_t)pair * I + blk * 128 + lane * 4, v);
                }
            }
        }
    }
}

template <int MODE, bool WIDE>
static int launch_pair_groups(const chronos_layer_t& L, const Plan& p, cudaStream_t st) {
    const size_t smem = MODE == 0 ? (size_t)kGroupPairs * (2 * L.inter + L.inter) * 4 : (size_t)kGroupPairs * L.hidden * 4;
    if (smem > 220 * 1024) {
        set_error("pair_group_out: %zu bytes of shared memory needed for hidden %d / inter %d", smem, L.hidden, L.inter);
        return CHRONOS_E_SHAPE;
    }
    const int sms = device_sm_count();
    const unsigned most = (unsigned)p.max_gitems * (unsigned)kGroupsPerItem;
    const unsigned resident = (unsigned)sms * (smem * 3 <= 225 * 1024 ? 3u : (smem * 2 <= 225 * 1024 ? 2u : 1u));
    const unsigned grid = most < resident ? most : resident;
    int rc = CHRONOS_OK;
#define CHRONOS_PG(R)                                                                                                   \
    rc = ensure_dynamic_smem(reinterpret_cast<const void*>(pair_group_out_kernel<MODE, R, WIDE>), smem, "pair_group_out"); \
    if (rc == CHRONOS_OK) pair_group_out_kernel<MODE, R, WIDE><<<grid, kOutThreads, smem, st>>>(L, p);
    switch (L.rank / 16) {
        case 1: CHRONOS_PG(1) break;
        case 2: CHRONOS_PG(2) break;
        case 4: CHRONOS_PG(4) break;
        default: CHRONOS_PG(8) break;
    }
#undef CHRONOS_PG
    if (rc != CHRONOS_OK) return rc;
    return check_launch("pair_group_out");
}

bool healer_mma_fits(const chronos_layer_t& L) {
    return L.v_dn != nullptr && (size_t)kGroupPairs * 3 * L.inter * 4 <= 220 * 1024 && (size_t)kGroupPairs * L.hidden * 4 <= 220 * 1024;
}

// The fused healer needs the FP4 tensor regime, the layer's healer tiles, a rank that fits a ring slot of the bank pass and
// shapes the gather kernels behind it serve (the regime's own limits imply them).
bool healer_fused(const chronos_layer_t& L, const Plan& p) {
    return p.fp4_wide && p.himg != nullptr && L.ut_gu != nullptr && L.ut_dn != nullptr && L.ut_scale != nullptr && L.rank <= 64 &&
           combine_gather_fits(L);
}

int launch_mid_mma(const chronos_layer_t& L, const Plan& p, int wide, cudaStream_t st) {
    const bool fused = wide && healer_fused(L, p);
    if (int rc = fused ? launch_mid_fused(L, p, st)
                       : (wide ? launch_pair_groups<0, true>(L, p, st) : launch_pair_groups<0, false>(L, p, st))) return rc;
    if (int rc = wide ? launch_healer_in_mma(L, 1, p.ac, kDtypeF16Scaled, p, st) : launch_healer_in_mma(L, 1, p.act, CHRONOS_DTYPE_F32, p, st)) return rc;
    return fused ? launch_heal_image(L, 1, p, st) : CHRONOS_OK;
}

int launch_down_out_mma(const chronos_layer_t& L, const Plan& p, cudaStream_t st) { return launch_pair_groups<1, false>(L, p, st); }

}  // namespace chronos
