// Tensor-core bank pass (prefill regime): for every work item (one expert, up to 128 of its sorted pairs) and every
// 128-row block of the slot's bank,
//     D[pair, row] = sum_k x_c[pair, k] * S[row, k]          (tcgen05.mma, fp32 accumulators in tensor memory)
//     z[pair, row-block] = H_128( r_s2 * scale_2 * D[pair, :] ) (epilogue: one thread owns a pair's 128 outputs)
//
// One persistent CTA per SM, 256 threads:
//   * all threads fill a ring of shared-memory stages: the activation tile (128 pairs x 64 columns, fp16) arrives by
//     cp.async, the bank tile (128 rows x 64 columns) is read as packed e2m1 nibbles + e4m3 block scales, converted
//     in registers (cvt.rn.f16x2.e2m1x2, one fp16 multiply by the block scale - exact) and stored as fp16; both
//     tiles use the K-major 128-byte-swizzled operand layout the MMA reads through shared-memory descriptors;
//   * thread 0 issues four 128x128x16 tcgen05.mma per stage and releases the stage with tcgen05.commit;
//   * after the K loop warps 0-3 pull the accumulator out of tensor memory (tcgen05.ld, thread t = TMEM lane t = pair
//     t), apply scale_2 and the expert's r_s2 signs, run the 128-point Walsh-Hadamard butterflies in registers and
//     store fp32 rows.
// The pairs sit on the MMA's M axis and the bank rows on N, so the Hadamard block of a pair is private to a thread.
// Every mbarrier wait is bounded; expiry raises the status word and the CTA drains.
#include "common.cuh"

namespace chronos {

constexpr int kGemmStages = 4;
constexpr int kGemmKStep = 64;                       // columns per stage (= one 128-byte swizzle row of fp16)
constexpr int kTileBytes = 128 * kGemmKStep * 2;     // one operand tile: 128 rows x 128 bytes
constexpr int kStatusGemmTimeout = kStatusBankGemmTimeout;
constexpr uint32_t kTmemCols = 128;

struct GemmArgs {
    const uint8_t* w; const uint8_t* s; const float* s2;
    const uint8_t* sh_w; const uint8_t* sh_s; const float* sh_s2; int sh_split;
    const uint32_t* rs2;
    const __half* xin;
    float* zout;
    const float* pscale;
    const int32_t* item_start; const int32_t* item_cnt; const int32_t* item_slot; const int32_t* pair_expert;
    int32_t* counters;
    int R, K, n_slots;
};

// K-major, 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart, 16-byte chunk index xor (row & 7).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void tc_mma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n.reg .pred p;\n"
        "setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
        "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

__global__ void __launch_bounds__(256, 1) bank_gemm_kernel(const GemmArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t bars[kGemmStages + 1];  // empty[S], accumulator-ready
    __shared__ uint32_t tmem_base_s;
    // operand tiles need 1024-byte alignment for the swizzle pattern to line up with the descriptor
    uint8_t* tiles = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);

    const int tid = threadIdx.x, warp = tid >> 5;
    const int R = a.R, K = a.K, RB = R / 128, KS = K / kGemmKStep;
    const long n_tiles = (long)a.counters[3] * RB;

    if (tid == 0) {
        for (int s = 0; s <= kGemmStages; ++s) mbar_init(smem_u32(&bars[s]), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {  // one warp allocates the accumulator columns and gives the permit back at once
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)), "r"(kTmemCols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_d = tmem_base_s;
    // instruction descriptor: D = f32, A = B = f16, both K-major, N = 128, M = 128
    const uint32_t idesc = (1u << 4) | ((128u >> 3) << 17) | ((128u >> 4) << 24);

    uint32_t it = 0, tile_count = 0;
    const int brow = tid >> 1, bhalf = tid & 1;  // bank-tile conversion: two threads per row, 32 nibbles each
    for (long tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++tile_count) {
        const int item = (int)(tile / RB), rb = (int)(tile % RB);
        const int start = a.item_start[item], cnt = a.item_cnt[item], slot = a.item_slot[item];
        const bool sh = slot >= a.n_slots;
        const uint8_t* wrow = (sh ? a.sh_w : a.w + (size_t)slot * R * (K / 2)) + ((size_t)rb * 128 + brow) * (K / 2) + bhalf * 16;
        const uint8_t* srow = (sh ? a.sh_s : a.s + (size_t)slot * R * (K / 16)) + ((size_t)rb * 128 + brow) * (K / 16) + bhalf * 2;
        uint4 nib = *reinterpret_cast<const uint4*>(wrow);
        uint16_t sc = *reinterpret_cast<const uint16_t*>(srow);
        bool aborted = false;
        for (int ks = 0; ks < KS; ++ks, ++it) {
            const int s = (int)(it % kGemmStages);
            const uint32_t ph = (it / kGemmStages) & 1u;
            const bool ok = mbar_wait(smem_u32(&bars[s]), ph ^ 1u);  // until the MMAs that read this stage are done
            uint8_t* sa = tiles + (size_t)s * 2 * kTileBytes;
            uint8_t* sb = sa + kTileBytes;
            // activation tile: 1024 chunks of 16 bytes, 4 per thread; rows past the item's pair count are zero-filled
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int c = tid + 256 * i, row = c >> 3, j = c & 7;
                const bool valid = row < cnt;
                const __half* src = a.xin + (size_t)(start + (valid ? row : 0)) * K + ks * kGemmKStep + j * 8;
                cp_async16(smem_u32(sa + row * 128 + ((j ^ (row & 7)) << 4)), src, valid ? 16u : 0u);
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
            // bank tile: convert this step's nibbles, prefetch the next step's
            const uint4 cur = nib;
            const uint16_t csc = sc;
            if (ks + 1 < KS) {
                nib = *reinterpret_cast<const uint4*>(wrow + (size_t)(ks + 1) * 32);
                sc = *reinterpret_cast<const uint16_t*>(srow + (size_t)(ks + 1) * 4);
            }
            uint32_t s2h;
            asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(s2h) : "h"(csc));
            const uint32_t sc0 = __byte_perm(s2h, 0, 0x1010), sc1 = __byte_perm(s2h, 0, 0x3232);
            const uint32_t wv[4] = {cur.x, cur.y, cur.z, cur.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {  // word q = nibbles 8q..8q+7 = one 16-byte chunk of fp16; scale block q / 2
                uint32_t h0, h1, h2, h3;
                e2m1x8_to_f16x2(wv[q], h0, h1, h2, h3);
                const uint32_t scl = q < 2 ? sc0 : sc1;
                uint4 o;
                o.x = hmul2_u32(h0, scl); o.y = hmul2_u32(h1, scl); o.z = hmul2_u32(h2, scl); o.w = hmul2_u32(h3, scl);
                const int j = bhalf * 4 + q;
                *reinterpret_cast<uint4*>(sb + brow * 128 + ((j ^ (brow & 7)) << 4)) = o;
            }
            asm volatile("cp.async.wait_group 0;" ::: "memory");
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic-proxy writes -> visible to the MMA
            if (__syncthreads_or(!ok)) {  // the same verdict in every thread
                aborted = true;
                break;
            }
            if (tid == 0) {
                tc_fence_after();
                const uint64_t da = smem_desc_sw128(smem_u32(sa)), db = smem_desc_sw128(smem_u32(sb));
#pragma unroll
                for (int kk = 0; kk < kGemmKStep / 16; ++kk)
                    tc_mma_f16(tmem_d, da + (uint64_t)(kk * 2), db + (uint64_t)(kk * 2), idesc, (ks > 0 || kk > 0) ? 1u : 0u);
                tc_commit(smem_u32(&bars[s]));
                if (ks == KS - 1) tc_commit(smem_u32(&bars[kGemmStages]));
            }
        }
        // ---- epilogue ----
        if (!aborted) aborted = __syncthreads_or(!mbar_wait(smem_u32(&bars[kGemmStages]), tile_count & 1u)) != 0;
        if (aborted) {
            if (tid == 0) atomicOr(a.counters + 2, kStatusGemmTimeout);
            break;
        }
        tc_fence_after();
        if (warp < 4) {
            float v[128];
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) {
                uint32_t r[32];
                tmem_ld32(tmem_d + ((uint32_t)(warp * 32) << 16) + (uint32_t)(c4 * 32), r);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int i = 0; i < 32; ++i) v[c4 * 32 + i] = __uint_as_float(r[i]);
            }
            if (tid < cnt) {
                const float s2 = (sh ? a.sh_s2[rb * 128 >= a.sh_split ? 1 : 0] : a.s2[slot]) * a.pscale[start + tid];
#pragma unroll
                for (int i = 0; i < 128; ++i) v[i] *= s2;
                if (!sh) {
                    const int e = a.pair_expert[start + tid];
                    const uint4 sg = *reinterpret_cast<const uint4*>(a.rs2 + (size_t)e * (R / 32) + rb * 4);
                    const uint32_t sw[4] = {sg.x, sg.y, sg.z, sg.w};
#pragma unroll
                    for (int i = 0; i < 128; ++i)
                        if ((sw[i >> 5] >> (i & 31)) & 1u) v[i] = -v[i];
#pragma unroll
                    for (int m = 1; m < 128; m <<= 1)
#pragma unroll
                        for (int i = 0; i < 128; ++i)
                            if ((i & m) == 0) {
                                const float x0 = v[i], x1 = v[i | m];
                                v[i] = x0 + x1;
                                v[i | m] = x0 - x1;
                            }
#pragma unroll
                    for (int i = 0; i < 128; ++i) v[i] *= 0.08838834764831845f;
                }
                float4* dst = reinterpret_cast<float4*>(a.zout + (size_t)(start + tid) * R + rb * 128);
#pragma unroll
                for (int i = 0; i < 32; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            }
        }
        tc_fence_before();
        __syncthreads();  // accumulator drained: the next tile may overwrite it
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(kTmemCols) : "memory");
}

int launch_bank_gemm(const chronos_layer_t& L, int stage, const Plan& p, cudaStream_t st) {
    GemmArgs a{};
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
    a.item_start = p.gitem_start;
    a.item_cnt = p.gitem_cnt;
    a.item_slot = p.gitem_slot;
    a.pair_expert = p.pair_expert;
    a.counters = p.counters;
    a.n_slots = L.n_slots;
    if (a.K % kGemmKStep) {
        set_error("bank_gemm: K = %d is not a multiple of %d", a.K, kGemmKStep);
        return CHRONOS_E_SHAPE;
    }
    const size_t smem = (size_t)kGemmStages * 2 * kTileBytes + 1024;
    if (int rc = ensure_dynamic_smem(reinterpret_cast<const void*>(bank_gemm_kernel), smem, "bank_gemm")) return rc;
    const int sms = device_sm_count();
    const long max_tiles = (long)p.max_gitems * (a.R / 128);
    const int grid = (int)(max_tiles < sms ? max_tiles : sms);
    bank_gemm_kernel<<<grid, 256, smem, st>>>(a);
    return check_launch("bank_gemm");
}

}  // namespace chronos
