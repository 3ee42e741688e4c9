// Streaming bank pass (HBM-bound regime): z[pair, row] = H_128-blocks( r_s2 * scale_2 * sum_k S[row, k] x_c[pair, k] )
// for up to 8 (token, expert) pairs per pass over a slot's packed NVFP4 bank, so every distinct slot is read once.
//
// Persistent kernel, one CTA per SM. Work tile = (work item, 128-row block of the bank).
//   * one producer warp streams the tile's packed rows (nibbles + e4m3 block scales) into a ring of shared-memory
//     stages with bulk async copies (cp.async.bulk, completion on an mbarrier) - 16 bank rows per stage;
//   * NW <= 8 consumer warps split K: warp w owns k-chunks [w*CPW, (w+1)*CPW) of 128 columns and keeps the matching
//     slice of the 8 transformed activation vectors in registers as m16n8k16 B fragments for the whole tile;
//   * per stage a consumer reads 2x16 bytes of nibbles per chunk, converts e2m1 -> f16x2 in hardware
//     (cvt.rn.f16x2.e2m1x2), multiplies by the e4m3 block scale (exact in fp16: 2-bit x 4-bit significands) and
//     issues 8 tensor-core MMAs with fp32 accumulation; k is permuted identically in A and B so that each lane's
//     16 contiguous bytes feed its own fragment slots with no shuffles;
//   * after 8 stages the per-warp partial sums are reduced in a fixed order through shared memory, scaled by
//     scale_2, signed by the pair's r_s2 key and pushed through the 128-point Walsh-Hadamard butterflies
//     (warp shuffles), then stored as fp32.
// Every mbarrier wait is bounded; on expiry the kernel raises the status word in the plan and drains.
#include "common.cuh"

namespace chronos {

constexpr int kRowsPerStage = 16;
constexpr int kStagesPerTile = 128 / kRowsPerStage;
constexpr int kRedStride = 132;           // floats per (warp, pair) row of the reduction buffer (bank-conflict pad)
constexpr int kStatusBankTimeout = kStatusBankStreamTimeout;

struct BankArgs {
    const uint8_t* w;       // [n_slots, R, K/2]
    const uint8_t* s;       // [n_slots, R, K/16]
    const float* s2;        // [n_slots]
    const uint8_t* sh_w;    // shared expert rows [R_sh_offset.., K/2] (slot == n_slots)
    const uint8_t* sh_s;
    const float* sh_s2;     // shared expert scale_2: [2] = (gate rows, up rows) in the gate_up pass, [1] in the down pass
    int sh_split;           // first row that uses sh_s2[1]
    const uint32_t* rs2;    // [E, R/32]
    const __half* xin;      // [P, K]
    float* zout;            // [P, R]
    const float* pscale;    // [P] power-of-two scale each pair's activation row was divided by
    const int32_t* item_start;
    const int32_t* item_cnt;
    const int32_t* item_slot;
    const int32_t* pair_expert;
    int32_t* counters;
    int R, K, n_slots, n_experts;
    int nib_stride, sc_stride, stage_bytes, n_stages, n_warps;
};

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void consumer_barrier(int n_threads) {
    asm volatile("bar.sync 1, %0;" ::"r"(n_threads) : "memory");
}

template <int CPW>
__global__ void __launch_bounds__(9 * 32, 1) bank_stream_kernel(const BankArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int NW = a.n_warps;       // consumer warps
    const int S = a.n_stages;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);  // full[S], empty[S]
    uint8_t* stage0 = smem + 256;
    float* red = reinterpret_cast<float*>(stage0 + (size_t)S * a.stage_bytes);  // [NW][8][kRedStride]
    __shared__ int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int R = a.R, K = a.K;
    const int RB = R / 128;
    const int n_chunks = K / 128;
    const long n_tiles = (long)a.counters[0] * RB;
    // each CTA takes a contiguous run of tiles: consecutive row blocks of one item share their B fragments
    const long tile_lo = n_tiles * blockIdx.x / gridDim.x, tile_hi = n_tiles * (blockIdx.x + 1) / gridDim.x;

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&bars[s]), 1);
            mbar_init(smem_u32(&bars[S + s]), (uint32_t)NW);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    const uint32_t stage_tx = (uint32_t)(kRowsPerStage * (K / 2 + K / 16));
    const int sc_off = kRowsPerStage * a.nib_stride;  // scales follow the nibble rows inside a stage

    if (warp == NW) {
        // ---------------- producer warp ----------------
        // Lane 0 runs the ring protocol; the row copies of a stage are issued by 32 lanes at once (lanes 0-15 one
        // nibble row each, lanes 16-31 one scale row each) because a single thread issues bulk copies too slowly
        // to keep HBM busy with 16 + 16 small copies per stage.
        uint32_t it = 0;
        bool live = true;
        const uint64_t pol = l2_policy_evict_first();
        for (long tile = tile_lo; tile < tile_hi && live; ++tile) {
            const int item = (int)(tile / RB), rb = (int)(tile % RB);
            const int slot = a.item_slot[item];
            const bool sh = slot >= a.n_slots;
            const uint8_t* wsrc = (sh ? a.sh_w : a.w + (size_t)slot * R * (K / 2)) + (size_t)rb * 128 * (K / 2);
            const uint8_t* ssrc = (sh ? a.sh_s : a.s + (size_t)slot * R * (K / 16)) + (size_t)rb * 128 * (K / 16);
            for (int rt = 0; rt < kStagesPerTile; ++rt, ++it) {
                const int s = (int)(it % (uint32_t)S);
                const uint32_t ph = (it / (uint32_t)S) & 1u;
                const uint32_t full = smem_u32(&bars[s]);
                int ok = 1;
                if (lane == 0) {
                    ok = mbar_wait(smem_u32(&bars[S + s]), ph ^ 1u) ? 1 : 0;
                    if (ok) mbar_expect_tx(full, stage_tx);
                    else atomicOr(a.counters + 2, kStatusBankTimeout);  // consumers stopped releasing stages
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) { live = false; break; }
                const uint32_t dst = smem_u32(stage0 + (size_t)s * a.stage_bytes);
                const uint8_t* wr = wsrc + (size_t)rt * kRowsPerStage * (K / 2);
                const uint8_t* sr = ssrc + (size_t)rt * kRowsPerStage * (K / 16);
                if (lane < 16) {
                    if (a.nib_stride == K / 2) {
                        if (lane == 0) bulk_g2s_stream(dst, wr, (uint32_t)(kRowsPerStage * (K / 2)), full, pol);
                    } else {
                        bulk_g2s_stream(dst + lane * a.nib_stride, wr + (size_t)lane * (K / 2), (uint32_t)(K / 2), full, pol);
                    }
                } else {
                    const int rr = lane - 16;
                    if (a.sc_stride == K / 16) {
                        if (rr == 0) bulk_g2s_stream(dst + sc_off, sr, (uint32_t)(kRowsPerStage * (K / 16)), full, pol);
                    } else {
                        bulk_g2s_stream(dst + sc_off + rr * a.sc_stride, sr + (size_t)rr * (K / 16), (uint32_t)(K / 16), full, pol);
                    }
                }
            }
        }
        // drain: every stage handed to the copy engine must land (or be consumed) before the CTA may exit
        if (lane == 0) {
            const uint32_t issued = it;
            for (uint32_t back = 0; back < (uint32_t)S && back < issued; ++back) {
                const uint32_t j = issued - 1 - back;
                if (!mbar_wait(smem_u32(&bars[j % (uint32_t)S]), (j / (uint32_t)S) & 1u)) {
                    atomicOr(a.counters + 2, kStatusBankTimeout);
                    break;
                }
            }
        }
        return;
    }
    if (warp > NW) return;

    // ---------------- consumer warps ----------------
    const int g = lane >> 2, q = lane & 3;
    const int consumer_threads = NW * 32;
    uint32_t it = 0;
    int cur_item = -1;
    uint32_t bfrag[CPW][16];
    for (long tile = tile_lo; tile < tile_hi; ++tile) {
        const int item = (int)(tile / RB), rb = (int)(tile % RB);
        const int start = a.item_start[item], cnt = a.item_cnt[item], slot = a.item_slot[item];
        const bool sh = slot >= a.n_slots;

        // B fragments: x_c[start + g][k-slice of this warp], 32 consecutive halves per chunk for lane (g, q);
        // kept across the row blocks of an item
        if (item != cur_item) {
        cur_item = item;
#pragma unroll
        for (int c = 0; c < CPW; ++c) {
            const int chunk = warp * CPW + c;
            if (g < cnt && chunk < n_chunks) {
                const uint4* src = reinterpret_cast<const uint4*>(a.xin + (size_t)(start + g) * K + chunk * 128 + q * 32);
#pragma unroll
                for (int v4 = 0; v4 < 4; ++v4) {
                    const uint4 t = src[v4];
                    bfrag[c][v4 * 4 + 0] = t.x; bfrag[c][v4 * 4 + 1] = t.y;
                    bfrag[c][v4 * 4 + 2] = t.z; bfrag[c][v4 * 4 + 3] = t.w;
                }
            } else {
#pragma unroll
                for (int v = 0; v < 16; ++v) bfrag[c][v] = 0u;
            }
        }
        }
        float acc[kStagesPerTile][4];
#pragma unroll
        for (int rt = 0; rt < kStagesPerTile; ++rt)
#pragma unroll
            for (int v = 0; v < 4; ++v) acc[rt][v] = 0.0f;

        bool live = true;
#pragma unroll
        for (int rt = 0; rt < kStagesPerTile; ++rt, ++it) {
            const int s = (int)(it % (uint32_t)S);
            const uint32_t ph = (it / (uint32_t)S) & 1u;
            if (live && !mbar_wait(smem_u32(&bars[s]), ph)) {
                atomicOr(a.counters + 2, kStatusBankTimeout);
                *(volatile int*)&abort_flag = 1;
                live = false;
            }
            if (live) {
                const uint8_t* st = stage0 + (size_t)s * a.stage_bytes;
#pragma unroll
                for (int c = 0; c < CPW; ++c) {
                    const int chunk = warp * CPW + c;
                    if (chunk < n_chunks) {
                        const uint4 lo = *reinterpret_cast<const uint4*>(st + g * a.nib_stride + chunk * 64 + q * 16);
                        const uint4 hi = *reinterpret_cast<const uint4*>(st + (g + 8) * a.nib_stride + chunk * 64 + q * 16);
                        const uint16_t sl = *reinterpret_cast<const uint16_t*>(st + sc_off + g * a.sc_stride + chunk * 8 + q * 2);
                        const uint16_t sh16 = *reinterpret_cast<const uint16_t*>(st + sc_off + (g + 8) * a.sc_stride + chunk * 8 + q * 2);
                        uint32_t sl2, sh2;  // (scale of block 0, scale of block 1) as f16x2
                        asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(sl2) : "h"(sl));
                        asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(sh2) : "h"(sh16));
                        const uint32_t sl_b0 = __byte_perm(sl2, 0, 0x1010), sl_b1 = __byte_perm(sl2, 0, 0x3232);
                        const uint32_t sh_b0 = __byte_perm(sh2, 0, 0x1010), sh_b1 = __byte_perm(sh2, 0, 0x3232);
                        const uint32_t low[4] = {lo.x, lo.y, lo.z, lo.w}, hiw[4] = {hi.x, hi.y, hi.z, hi.w};
#pragma unroll
                        for (int wq = 0; wq < 4; ++wq) {
                            // word wq = bytes 4wq..4wq+3 = nibbles 8wq..8wq+7 -> scale block wq / 2
                            uint32_t l0, l1, l2, l3, h0, h1, h2, h3;
                            e2m1x8_to_f16x2(low[wq], l0, l1, l2, l3);
                            e2m1x8_to_f16x2(hiw[wq], h0, h1, h2, h3);
                            const uint32_t sL = wq < 2 ? sl_b0 : sl_b1, sH = wq < 2 ? sh_b0 : sh_b1;
                            // MMA 2wq uses bytes 0,1 of the word; MMA 2wq+1 uses bytes 2,3
                            mma_f16(acc[rt], hmul2_u32(l0, sL), hmul2_u32(h0, sH), hmul2_u32(l1, sL), hmul2_u32(h1, sH),
                                    bfrag[c][wq * 4 + 0], bfrag[c][wq * 4 + 1]);
                            mma_f16(acc[rt], hmul2_u32(l2, sL), hmul2_u32(h2, sH), hmul2_u32(l3, sL), hmul2_u32(h3, sH),
                                    bfrag[c][wq * 4 + 2], bfrag[c][wq * 4 + 3]);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&bars[S + s]));
        }

        // ---- epilogue: fixed-order cross-warp reduction, scale_2, r_s2 sign, 128-point WHT over the rows ----
        float* my = red + (size_t)warp * 8 * kRedStride;
#pragma unroll
        for (int rt = 0; rt < kStagesPerTile; ++rt) {
            my[(2 * q) * kRedStride + rt * 16 + g] = acc[rt][0];
            my[(2 * q + 1) * kRedStride + rt * 16 + g] = acc[rt][1];
            my[(2 * q) * kRedStride + rt * 16 + g + 8] = acc[rt][2];
            my[(2 * q + 1) * kRedStride + rt * 16 + g + 8] = acc[rt][3];
        }
        consumer_barrier(consumer_threads);
        const float s2 = sh ? a.sh_s2[rb * 128 >= a.sh_split ? 1 : 0] : a.s2[slot];
        for (int n = warp; n < cnt; n += NW) {
            float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int ww = 0; ww < NW; ++ww) {
                const float4 t = *reinterpret_cast<const float4*>(red + ((size_t)ww * 8 + n) * kRedStride + lane * 4);
                v[0] += t.x; v[1] += t.y; v[2] += t.z; v[3] += t.w;
            }
            const float sc = s2 * a.pscale[start + n];
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] *= sc;
            if (!sh) {
                const int e = a.pair_expert[start + n];
                const uint32_t sw = a.rs2[(size_t)e * (R / 32) + rb * 4 + lane / 8] >> ((lane & 7) * 4);
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if ((sw >> i) & 1u) v[i] = -v[i];
                fwht128_warp(v, lane);
            }
            *reinterpret_cast<float4*>(a.zout + (size_t)(start + n) * R + rb * 128 + lane * 4) =
                make_float4(v[0], v[1], v[2], v[3]);
        }
        consumer_barrier(consumer_threads);
        if (!live || *(volatile int*)&abort_flag) break;
    }
}

// k-chunks of 128 columns per consumer warp: at most 8 consumer warps, at most 8 chunks each (K <= 8192)
static int pick_cpw(int n_chunks) {
    const int cpw = (n_chunks + 7) / 8;
    return cpw <= 8 ? cpw : 0;
}

int launch_bank_stream(const chronos_layer_t& L, int stage, const Plan& p, cudaStream_t st) {
    BankArgs a{};
    a.K = stage == 0 ? L.hidden : L.inter;
    a.R = stage == 0 ? 2 * L.inter : L.hidden;
    a.w = stage == 0 ? L.gu_w : L.dn_w;
    a.s = stage == 0 ? L.gu_s : L.dn_s;
    a.s2 = stage == 0 ? L.gu_s2 : L.dn_s2;
    a.sh_w = stage == 0 ? L.sh_gu_w : L.sh_dn_w;
    a.sh_s = stage == 0 ? L.sh_gu_s : L.sh_dn_s;
    a.sh_s2 = stage == 0 ? L.sh_gu_s2 : L.sh_dn_s2;
    a.sh_split = stage == 0 ? L.inter : 0x7fffffff;
    a.rs2 = stage == 0 ? L.gu_rs2 : L.dn_rs2;
    a.xin = stage == 0 ? p.xc : p.ac;
    a.zout = stage == 0 ? p.z1 : p.y1;
    a.pscale = stage == 0 ? p.pscale_gu : p.pscale_dn;
    a.item_start = p.item_start;
    a.item_cnt = p.item_cnt;
    a.item_slot = p.item_slot;
    a.pair_expert = p.pair_expert;
    a.counters = p.counters;
    a.n_slots = L.n_slots;
    a.n_experts = L.n_experts;
    const int n_chunks = a.K / 128;
    const int cpw = pick_cpw(n_chunks);
    if (cpw == 0) {
        set_error("bank_stream: K = %d exceeds the 8192 columns the streaming kernel supports", a.K);
        return CHRONOS_E_SHAPE;
    }
    a.n_warps = (n_chunks + cpw - 1) / cpw;
    a.nib_stride = a.K / 2 + (((a.K / 2) % 128 == 0) ? 64 : 0);
    a.sc_stride = a.K / 16 + (((a.K / 16) % 16 == 0) ? 16 : 0);
    a.stage_bytes = (int)align_up((size_t)kRowsPerStage * (a.nib_stride + a.sc_stride), 128);
    const size_t red_bytes = (size_t)a.n_warps * 8 * kRedStride * sizeof(float);
    const size_t budget = 220 * 1024;
    int stages = (int)((budget - 256 - red_bytes) / (size_t)a.stage_bytes);
    if (stages > 8) stages = 8;
    if (stages < 2) {
        set_error("bank_stream: a stage of %d bytes does not fit twice in shared memory", a.stage_bytes);
        return CHRONOS_E_SHAPE;
    }
    a.n_stages = stages;
    const size_t smem = 256 + (size_t)stages * a.stage_bytes + red_bytes;

    const int sms = device_sm_count();
    const long max_tiles = (long)p.max_items * (a.R / 128);
    const int grid = (int)(max_tiles < sms ? max_tiles : sms);
    const int threads = (a.n_warps + 1) * 32;

    auto go = [&](auto kern) -> int {
        if (int rc = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), smem, "bank_stream")) return rc;
        kern<<<grid, threads, smem, st>>>(a);
        return check_launch("bank_stream");
    };
    switch (cpw) {
        case 1: return go(bank_stream_kernel<1>);
        case 2: return go(bank_stream_kernel<2>);
        case 3: return go(bank_stream_kernel<3>);
        case 4: return go(bank_stream_kernel<4>);
        case 5: return go(bank_stream_kernel<5>);
        case 6: return go(bank_stream_kernel<6>);
        case 7: return go(bank_stream_kernel<7>);
        default: return go(bank_stream_kernel<8>);
    }
}

}  // namespace chronos
