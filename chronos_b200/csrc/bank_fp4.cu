// Block-scaled FP4 tensor-core path: tcgen05.mma kind::mxf4nvf4 (e2m1 operands, ue4m3 scale per 16 elements).
//
// Operand images. A "stage" covers 256 columns (K) = four MMAs of K = 64.
//   matrix tile of R rows x 256 columns, packed e2m1 (two per byte, lower column in the low nibble):
//       byte(r, c, b) at c * (R * 16) + r * 16 + b        c = 16-byte chunk 0..7 along K, b = byte in chunk
//     i.e. the K-major "interleaved" (no swizzle) operand layout: 8-row x 16-byte core matrices, rows 16 B apart,
//     8-row groups 128 B apart (SBO), neighbouring K chunks R*16 B apart (LBO).
//   scale factors of the tile: four 512-byte blocks (one per MMA), block j byte(r, s) at (r % 32) * 16 + (r / 32) * 4 + s
//     with s = 16-column block 0..3 inside the MMA's 64 columns: the layout tcgen05.cp 32x128b.warpx4 moves into
//     tensor memory (lane = r % 32, 32-bit column = r / 32, byte = s).
// The bank side (128 rows) is re-tiled once at load from the on-disk row-major bytes: 16384 B of nibbles followed by
// 2048 B of scales per (slot, 128-row block, stage), so one bulk copy fetches a whole stage. The activation side
// (32 rows: 8 pairs x 3 residual terms, padded) is written in the same format by the quantiser kernels.
#include "common.cuh"

namespace chronos {

constexpr int kF4StageK = 256;                       // columns per stage
constexpr int kF4ARows = 128;                        // bank rows per tile (MMA M)
constexpr int kF4BRows = 32;                         // activation rows per tile (MMA N): 8 pairs x 3 terms + padding
constexpr int kF4ANib = kF4ARows * kF4StageK / 2;    // 16384
constexpr int kF4BNib = kF4BRows * kF4StageK / 2;    // 4096
constexpr int kF4SfBytes = 4 * 512;                  // scale blocks of one stage
constexpr int kF4AStage = kF4ANib + kF4SfBytes;      // 18432
constexpr int kF4BStage = kF4BNib + kF4SfBytes;      // 6144

// K-major, no swizzle: leading-dimension (K) byte offset between 16-byte chunks, stride (row-group) byte offset 128.
__device__ __forceinline__ uint64_t smem_desc_interleaved(uint32_t saddr, uint32_t lbo_bytes) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16) | ((uint64_t)(128u >> 4) << 32) |
           (1ull << 46);
}

__device__ __forceinline__ void tc_cp_sf(uint32_t tmem_dst, uint32_t smem_src) {
    // 32 rows x 16 bytes (one 512-byte scale block) -> 4 tensor-memory columns, replicated to the 4 lane quarters
    const uint64_t desc = (uint64_t)((smem_src >> 4) & 0x3FFFu) | ((uint64_t)(128u >> 4) << 32) | (1ull << 46);
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(tmem_dst), "l"(desc) : "memory");
}

__device__ __forceinline__ void tc_mma_nvf4(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t sfa,
                                            uint32_t sfb, uint32_t accumulate) {
    asm volatile(
        "{\n.reg .pred p;\n"
        "setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n}\n" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
        : "memory");
}

__device__ __forceinline__ void tc_commit_f4(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_ld32_f4(uint32_t taddr, uint32_t (&r)[32]) {
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

__device__ __forceinline__ void tmem_ld16_f4(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}

// Lean forms for the issuing thread (its instruction stream is the critical path of the streaming kernel): the
// descriptors' high words are constants, the low words are a base plus a 16-byte-unit offset.
__device__ __forceinline__ void tc_cp_sf_lo(uint32_t tmem_dst, uint32_t desc_lo) {
    asm volatile("{\n.reg .b64 d;\nmov.b64 d, {%1, %2};\ntcgen05.cp.cta_group::1.32x128b.warpx4 [%0], d;\n}" ::"r"(tmem_dst),
                 "r"(desc_lo), "r"(0x00004008u)
                 : "memory");
}
template <bool ACC>
__device__ __forceinline__ void tc_mma_nvf4_lo(uint32_t tmem_d, uint32_t da_lo, uint32_t da_hi, uint32_t db_lo, uint32_t db_hi,
                                               uint32_t idesc, uint32_t sfa, uint32_t sfb) {
    if (ACC)
        asm volatile(
            "{\n.reg .b64 a, b;\n.reg .pred p;\nmov.b64 a, {%1, %2};\nmov.b64 b, {%3, %4};\nsetp.eq.u32 p, 0, 0;\n"
            "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], a, b, %5, [%6], [%7], p;\n}" ::"r"(tmem_d),
            "r"(da_lo), "r"(da_hi), "r"(db_lo), "r"(db_hi), "r"(idesc), "r"(sfa), "r"(sfb)
            : "memory");
    else
        asm volatile(
            "{\n.reg .b64 a, b;\n.reg .pred p;\nmov.b64 a, {%1, %2};\nmov.b64 b, {%3, %4};\nsetp.ne.u32 p, 0, 0;\n"
            "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], a, b, %5, [%6], [%7], p;\n}" ::"r"(tmem_d),
            "r"(da_lo), "r"(da_hi), "r"(db_lo), "r"(db_hi), "r"(idesc), "r"(sfa), "r"(sfb)
            : "memory");
}

// instruction descriptor, block-scaled: A = B = e2m1 (code 1), K-major, scale format ue4m3 (0), N at [17,23), M at [24,29)
__device__ __forceinline__ uint32_t idesc_nvf4(int m, int n) {
    return (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// ---------------------------------------------------------------------------------------------------------------
// Operand-format probe: D[128, NB] = sum over n_stages * 256 columns of (A * scaleA) (B * scaleB)^T, one CTA.
// a_img: n_stages x 18432 B; b_img: n_stages x (NB * 128 + 2048 * ceil(NB / 128)) B in the layouts above, NB = 32
// (streaming regime) ... 256 rows in steps of 16. Used by the parity tests to pin the descriptor, scale-factor and
// nibble conventions against a plain dequantise-and-multiply on the CPU.
// ---------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(128, 1) fp4_mma_probe_kernel(const uint8_t* __restrict__ a_img,
                                                               const uint8_t* __restrict__ b_img, int n_stages, int nb,
                                                               float* __restrict__ d_out, int32_t* __restrict__ status) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t bars[2];  // stage landed, MMAs done
    __shared__ uint32_t tmem_base_s;
    uint8_t* sa = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* sb = sa + kF4AStage;  // 18432 is a multiple of 1024
    const int tid = threadIdx.x, warp = tid >> 5;
    const int nblk = (nb + 127) / 128;                 // 512-byte scale blocks per MMA on the B side
    const uint32_t b_nib = (uint32_t)nb * 128u, b_stage = b_nib + 2048u * nblk;
    if (tid == 0) {
        mbar_init(smem_u32(&bars[0]), 1);
        mbar_init(smem_u32(&bars[1]), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)), "r"(512u) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base_s;
    const uint32_t tmem_d = tmem, tmem_sfa = tmem + 256, tmem_sfb = tmem + 272;  // 256 + 16 + up to 32 columns
    const uint32_t idesc = idesc_nvf4(kF4ARows, nb);
    int failed = 0;
    for (int st = 0; st < n_stages && !failed; ++st) {
        if (tid == 0) {
            mbar_expect_tx(smem_u32(&bars[0]), kF4AStage + b_stage);
            bulk_g2s(smem_u32(sa), a_img + (size_t)st * kF4AStage, kF4AStage, smem_u32(&bars[0]));
            bulk_g2s(smem_u32(sb), b_img + (size_t)st * b_stage, b_stage, smem_u32(&bars[0]));
            bool ok = mbar_wait(smem_u32(&bars[0]), st & 1);
            if (ok) {
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    tc_cp_sf(tmem_sfa + 4 * j, smem_u32(sa + kF4ANib + 512 * j));
                    for (int k = 0; k < nblk; ++k)
                        tc_cp_sf(tmem_sfb + 4 * nblk * j + 4 * k, smem_u32(sb + b_nib + 512 * (nblk * j + k)));
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint64_t da = smem_desc_interleaved(smem_u32(sa + 2 * j * (kF4ARows * 16)), kF4ARows * 16);
                    const uint64_t db = smem_desc_interleaved(smem_u32(sb + 2 * j * (nb * 16)), nb * 16);
                    tc_mma_nvf4(tmem_d, da, db, idesc, tmem_sfa + 4 * j, tmem_sfb + 4 * nblk * j, (st > 0 || j > 0) ? 1u : 0u);
                }
                tc_commit_f4(smem_u32(&bars[1]));
                ok = mbar_wait(smem_u32(&bars[1]), st & 1);  // single-buffered: wait before the next stage overwrites
            }
            if (!ok) atomicOr(status, kStatusFp4ProbeTimeout);
        }
        failed = __syncthreads_or(tid == 0 ? (*(volatile int32_t*)status != 0) : 0);
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (!failed) {
        for (int c0 = 0; c0 < nb; c0 += 16) {
            uint32_t r[16];
            tmem_ld16_f4(tmem_d + (uint32_t)c0 + ((uint32_t)(warp * 32) << 16), r);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
            for (int i = 0; i < 16; ++i) d_out[(size_t)tid * nb + c0 + i] = __uint_as_float(r[i]);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u) : "memory");
}

// ---------------------------------------------------------------------------------------------------------------
// Streaming bank pass on the block-scaled FP4 tensor cores (decode regime): no conversion work on the CUDA cores.
//   z[pair, row] = H_128-blocks( r_s2 * scale_2 * g_pair * sum_t 32^-t * D[row, t*8 + p] ),
//   D = (bank tile, e2m1 x ue4m3 as stored) x (activation image: 8 pairs x 3 residual e2m1 terms)^T.
// Persistent, one CTA per SM, 6 warps:
//   warp 0    producer: per stage two bulk copies (18432 B of re-tiled bank, 6144 B of activation image) into a ring;
//   warp 1    MMA issuer: per stage 8 scale-block copies to tensor memory (tcgen05.cp) and 4 tcgen05.mma of
//             128 x 32 x 64; tcgen05.commit frees the stage; two accumulator buffers in tensor memory;
//   warps 2-5 epilogue: tcgen05.ld (thread = bank row), combine the 3 terms, scale, then per pair r_s2 sign and the
//             128-point Walsh-Hadamard butterflies over the rows (shared-memory transpose + warp shuffles).
// Every mbarrier wait is bounded; on expiry the role raises the status word and stops, the others run into their
// own bounded waits.
// ---------------------------------------------------------------------------------------------------------------
constexpr int kF4MaxStages = 8;
constexpr int kF4Threads = 224;  // producer, MMA issuer A, 4 epilogue warps, MMA issuer B
constexpr int kF4SideThreads = 128;  // fused decode path: 4 more warps for the healer product of the pass
constexpr int kStatusFp4Timeout = kStatusBankFp4Timeout;
constexpr uint32_t kF4TmemCols = 512;  // 2 buffers x 2 accumulators x 32 columns, then bank scales (16 per ring stage), then activation scales

// Healer product the side warps of the fused decode path compute while the bank streams (kind 0: none).
//   kind 1 (gate_up pass): heal[pair, row] = g_pair * U_gu[e, row, :] . (V_gu[e] . x[token(pair), :] / g),  g = token scale
//   kind 2 (down pass):    heal[pair, row] = g_pair * U_down[e, row, :] . (V_down[e] . ac[pair, :]),  ac = act / g
// per chunk of up to 8 sorted pairs of one expert, on mma.sync m16n8k16 (e4m3 factors converted to fp16 exactly).
struct Fp4Side {
    int kind;
    const uint8_t* u;          // [E, R, r]
    const uint8_t* v;          // input factor [E, r, kc]: healer.v_gu (kind 1) / healer.v_down as on disk (kind 2)
    const void* x; int x_dtype; const int32_t* pair_token;  // kind 1: activation rows [T, kc] (bf16 / fp32)
    const __half* ac;          // kind 2: [P, kc]
    const float* pscale;       // [P]
    float* heal;               // [P, R]
    const int32_t* chunk_start; const int32_t* chunk_cnt;
    int rank, n_experts, kc;   // kc: contraction length of the input product (H for kind 1, I for kind 2)
};

struct Fp4Args {
    Fp4Side side;
    const uint8_t* bank_t;     // [n_slots, RB, NS, 18432]
    const uint8_t* sh_bank_t;  // [RB, NS, 18432] shared expert (slot == n_slots)
    const float* s2; const float* sh_s2; int sh_split;
    const uint32_t* rs2;
    const uint8_t* bq;         // [items, NS, 6144]
    const float* pscale;       // [P]
    float* zout;               // [P, R]
    const int32_t* item_start; const int32_t* item_cnt; const int32_t* item_slot; const int32_t* pair_expert;
    int32_t* counters;
    int R, K, n_slots, n_stages;
    int split_tiles;           // the output rows start at zero (fused decode path): tiles may be split between two CTAs
};

// The side warps' work (4 warps = one team per CTA; tasks are dealt round-robin over the CTAs). Every step requests the
// healer bytes of several tiles before multiplying any: the work is a handful of dependent round trips to L2 / HBM, and
// the number of requests in flight is what bounds it.
template <int R16>
__device__ __forceinline__ void side_healer(const Fp4Args& a, __half (*hsm)[kMaxRank], int sw, int lane) {
    const Fp4Side& sd = a.side;
    constexpr int r = R16 * 16;
    constexpr int G = R16 >= 8 ? 4 : 8;  // 16-row tiles whose rows are requested together (64 registers of healer bytes)
    const int g = lane >> 2, q = lane & 3;
    const int R = a.R, n_chunks = a.counters[3];
    if (n_chunks <= 0) return;
    const int n_tiles16 = R / 16;
    // chunks are few (one per distinct expert, about): when there are CTAs to spare a chunk's output rows are cut into
    // slices handled by different CTAs (each recomputes the chunk's small input product)
    int n_slices = (int)gridDim.x / n_chunks;
    n_slices = n_slices < 1 ? 1 : (n_slices > 8 ? 8 : n_slices);
    const int tiles_per_slice = (n_tiles16 + n_slices - 1) / n_slices;
    for (int task = blockIdx.x; task < n_chunks * n_slices; task += gridDim.x) {
        const int ch = task / n_slices, slice = task % n_slices;
        const int start = sd.chunk_start[ch], cnt = sd.chunk_cnt[ch];
        const int e = a.pair_expert[start];
        if (e >= sd.n_experts) continue;  // shared expert: no healer (uniform over the team)
        asm volatile("bar.sync 3, 128;" ::: "memory");  // the previous chunk's factors are no longer read
        {
            // h[n, c] = sum_k V[e, c, k] * a[pair n, k] with a = x[token] / g (kind 1) or ac[pair] (kind 2): warp sw takes the
            // 16-row tiles sw, sw + 4, ...; four 64-column steps of both operands are requested before they are multiplied.
            // Lane (g, q) owns a contiguous run of 16 columns per step on both operands (any permutation of the contraction
            // index is legal when both operands use it).
            const bool valid = g < cnt;
            const int prow = start + (valid ? g : 0);
            const uint8_t* arow;
            float inv = 0.0f;
            int abytes = 2;
            if (sd.kind == 1) {
                abytes = sd.x_dtype == CHRONOS_DTYPE_F32 ? 4 : 2;
                arow = reinterpret_cast<const uint8_t*>(sd.x) + ((size_t)sd.pair_token[prow] * sd.kc + 16 * q) * abytes;
                inv = valid ? 1.0f / sd.pscale[prow] : 0.0f;
            } else {
                arow = reinterpret_cast<const uint8_t*>(sd.ac + (size_t)prow * sd.kc + 16 * q);
            }
            for (int mt = sw; mt < R16; mt += 4) {
                const uint8_t* v0 = sd.v + ((size_t)e * r + mt * 16 + g) * sd.kc + 16 * q;
                const uint8_t* v1 = v0 + (size_t)8 * sd.kc;
                float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                // eight 64-column steps of the healer factor are requested at once (the bytes come from HBM); the activations
                // of a step are fetched one step ahead (a few rows shared by the team's warps: they stay in L1)
                auto load_act = [&](int kc, uint32_t (&bf)[8]) {
                    kc = min(kc, sd.kc - 64);
                    if (sd.kind == 2) {
                        uint4 u0 = make_uint4(0u, 0u, 0u, 0u), u1 = u0;
                        if (valid) {
                            u0 = *reinterpret_cast<const uint4*>(arow + (size_t)kc * 2);
                            u1 = *reinterpret_cast<const uint4*>(arow + (size_t)kc * 2 + 16);
                        }
                        bf[0] = u0.x; bf[1] = u0.y; bf[2] = u0.z; bf[3] = u0.w; bf[4] = u1.x; bf[5] = u1.y; bf[6] = u1.z; bf[7] = u1.w;
                    } else if (abytes == 2) {
                        const uint4 u0 = *reinterpret_cast<const uint4*>(arow + (size_t)kc * 2);
                        const uint4 u1 = *reinterpret_cast<const uint4*>(arow + (size_t)kc * 2 + 16);
                        const uint32_t uu[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            bf[j] = pack_f16x2_sat(__uint_as_float(uu[j] << 16) * inv, __uint_as_float(uu[j] & 0xffff0000u) * inv);
                    } else {
                        const float4* src = reinterpret_cast<const float4*>(arow + (size_t)kc * 4);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float4 f = src[j];
                            bf[2 * j] = pack_f16x2_sat(f.x * inv, f.y * inv);
                            bf[2 * j + 1] = pack_f16x2_sat(f.z * inv, f.w * inv);
                        }
                    }
                };
                for (int kc0 = 0; kc0 < sd.kc; kc0 += 512) {
                    uint4 w0[8], w1[8];
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const int kc = kc0 + 64 * c;
                        w0[c] = w1[c] = make_uint4(0u, 0u, 0u, 0u);  // steps past the end multiply zero healer bytes
                        if (kc < sd.kc) {
                            w0[c] = *reinterpret_cast<const uint4*>(v0 + kc);
                            w1[c] = *reinterpret_cast<const uint4*>(v1 + kc);
                        }
                    }
                    uint32_t bf[8], bn[8];
                    load_act(kc0, bf);
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        if (c + 1 < 8) load_act(kc0 + 64 * (c + 1), bn);
                        const uint32_t r0[4] = {w0[c].x, w0[c].y, w0[c].z, w0[c].w}, r1[4] = {w1[c].x, w1[c].y, w1[c].z, w1[c].w};
#pragma unroll
                        for (int s4 = 0; s4 < 4; ++s4)
                            mma_16816(acc, e4m3x2_to_f16x2(r0[s4] & 0xffffu), e4m3x2_to_f16x2(r1[s4] & 0xffffu), e4m3x2_to_f16x2(r0[s4] >> 16),
                                      e4m3x2_to_f16x2(r1[s4] >> 16), bf[2 * s4], bf[2 * s4 + 1]);
#pragma unroll
                        for (int j = 0; j < 8; ++j) bf[j] = bn[j];
                    }
                }
#pragma unroll
                for (int j = 0; j < 4; ++j)  // acc[j]: rank row mt*16 + g (+ 8), pair 2q + (j & 1)
                    hsm[2 * q + (j & 1)][mt * 16 + g + (j >> 1) * 8] = f32_to_f16_sat(acc[j]);
            }
        }
        asm volatile("bar.sync 3, 128;" ::: "memory");
        // B fragments: h[pair g][4 R16 q + 4 s .. + 3] as two fp16 pairs per k16 step
        uint32_t bf[R16][2];
#pragma unroll
        for (int s4 = 0; s4 < R16; ++s4) {
            const uint2 hv = *reinterpret_cast<const uint2*>(&hsm[g][4 * R16 * q + 4 * s4]);
            bf[s4][0] = hv.x;
            bf[s4][1] = hv.y;
        }
        const float gs0 = 2 * q < cnt ? sd.pscale[start + 2 * q] : 0.0f, gs1 = 2 * q + 1 < cnt ? sd.pscale[start + 2 * q + 1] : 0.0f;
        const uint8_t* U = sd.u + (size_t)e * R * r;
        const int t_lo = slice * tiles_per_slice, t_hi = min(n_tiles16, t_lo + tiles_per_slice);
        for (int jt0 = t_lo + sw * G; jt0 < t_hi; jt0 += 4 * G) {
            uint32_t wl[G][R16], wh[G][R16];
#pragma unroll
            for (int t = 0; t < G; ++t) {
                const int jt = jt0 + t;
                if (jt < t_hi) {
                    const uint32_t* u_lo = reinterpret_cast<const uint32_t*>(U + (size_t)(jt * 16 + g) * r + 4 * R16 * q);
                    const uint32_t* u_hi = reinterpret_cast<const uint32_t*>(U + (size_t)(jt * 16 + g + 8) * r + 4 * R16 * q);
                    if constexpr (R16 % 4 == 0) {
#pragma unroll
                        for (int s4 = 0; s4 < R16; s4 += 4) {
                            const uint4 a4 = *reinterpret_cast<const uint4*>(u_lo + s4), b4 = *reinterpret_cast<const uint4*>(u_hi + s4);
                            wl[t][s4] = a4.x; wl[t][s4 + 1] = a4.y; wl[t][s4 + 2] = a4.z; wl[t][s4 + 3] = a4.w;
                            wh[t][s4] = b4.x; wh[t][s4 + 1] = b4.y; wh[t][s4 + 2] = b4.z; wh[t][s4 + 3] = b4.w;
                        }
                    } else {
#pragma unroll
                        for (int s4 = 0; s4 < R16; ++s4) { wl[t][s4] = u_lo[s4]; wh[t][s4] = u_hi[s4]; }
                    }
                }
            }
#pragma unroll
            for (int t = 0; t < G; ++t) {
                const int jt = jt0 + t;
                if (jt < t_hi) {
                    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                    for (int s4 = 0; s4 < R16; ++s4)
                        mma_16816(d, e4m3x2_to_f16x2(wl[t][s4] & 0xffffu), e4m3x2_to_f16x2(wh[t][s4] & 0xffffu), e4m3x2_to_f16x2(wl[t][s4] >> 16),
                                  e4m3x2_to_f16x2(wh[t][s4] >> 16), bf[s4][0], bf[s4][1]);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {  // d[j]: row jt*16 + g (+ 8 for j >= 2), pair 2q + (j & 1)
                        const int n = 2 * q + (j & 1), row = jt * 16 + g + (j >> 1) * 8;
                        if (n < cnt) sd.heal[(size_t)(start + n) * R + row] = ((j & 1) ? gs1 : gs0) * d[j];
                    }
                }
            }
        }
    }
}

// Shared memory: [activation image of the current work item: NS x 6144 B][ring of n_stages bank stages x 18432 B].
// The activation image is fetched once per work item and stays while the CTA walks the item's row blocks
// (a CTA owns a contiguous run of tiles, so it changes item only once or twice per launch).
template <bool SIDE>
__global__ void __launch_bounds__(kF4Threads + (SIDE ? kF4SideThreads : 0), 1) bank_fp4_kernel(const Fp4Args a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t bars[2 * kF4MaxStages + 6];  // full[S], empty[S], acc_full[2], acc_empty[2], b_full, b_empty
    __shared__ uint32_t tmem_base_s;
    __shared__ __align__(16) float zs[2][8][128];    // epilogue exchange between the four lane quarters, double-buffered
    __shared__ __align__(16) __half hsm[SIDE ? 8 : 1][kMaxRank];  // side warps: healer input factors of the current chunk
    uint8_t* bimg = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int R = a.R, RB = R / 128, NS = a.K / kF4StageK, S = a.n_stages;
    uint8_t* stages = bimg + (size_t)NS * kF4BStage;  // 6144 * NS is a multiple of 1024 when NS is even; descriptors need 16 B only
    // Work split. A tile = (work item, 128-row block) = NS stages. Whole tiles per CTA leave the CTAs that get one tile more
    // than the others running alone at the end (9 or 10 tiles each is a 10 % tail). With `split_tiles` the launch's stage
    // sequence is cut into equal runs instead: a CTA's first and last tile may be partial (a slice of the contraction), and
    // the two CTAs that share a tile add their halves into the zero-initialised output (two addends: the sum does not
    // depend on their order).
    const long n_tiles = (long)a.counters[0] * RB;
    const long total_st = n_tiles * NS;
    long s_lo, s_hi;
    if (a.split_tiles && total_st / (long)gridDim.x >= NS) {
        s_lo = total_st * blockIdx.x / gridDim.x;
        s_hi = total_st * (blockIdx.x + 1) / gridDim.x;
    } else {
        s_lo = (n_tiles * blockIdx.x / gridDim.x) * NS;
        s_hi = (n_tiles * (blockIdx.x + 1) / gridDim.x) * NS;
    }
    const long tile_lo = s_lo / NS, tile_hi = s_hi > s_lo ? (s_hi - 1) / NS + 1 : tile_lo;  // tiles [tile_lo, tile_hi)
    auto st_begin = [&](long tile) { return tile == tile_lo ? (int)(s_lo % NS) : 0; };
    auto st_end = [&](long tile) { return tile == tile_hi - 1 ? (int)((s_hi - 1) % NS) + 1 : NS; };
    uint64_t* full = bars;
    uint64_t* empty = bars + kF4MaxStages;
    uint64_t* acc_full = bars + 2 * kF4MaxStages;
    uint64_t* acc_empty = bars + 2 * kF4MaxStages + 2;
    uint64_t* b_full = bars + 2 * kF4MaxStages + 4;
    uint64_t* b_empty = bars + 2 * kF4MaxStages + 5;
    // two issuing threads take the even / odd stages of every tile into separate accumulators (the issuing thread's
    // instruction stream is the critical path); activation scales too large to stay in TMEM keep one issuer
    const bool sfb_resident = 128 + S * 16 + NS * 16 <= (int)kF4TmemCols;  // activation scales of a whole item fit in TMEM
    const uint32_t n_issuers = sfb_resident ? 2u : 1u;

    if (tid == 0) {
        for (int s = 0; s < kF4MaxStages; ++s) { mbar_init(smem_u32(&full[s]), 1); mbar_init(smem_u32(&empty[s]), 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(smem_u32(&acc_full[b]), n_issuers); mbar_init(smem_u32(&acc_empty[b]), 4); }
        mbar_init(smem_u32(b_full), 1);
        mbar_init(smem_u32(b_empty), n_issuers);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)), "r"(kF4TmemCols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base_s;
    const uint32_t tmem_sf0 = tmem + 128;  // bank scales: 16 columns per ring stage; activation scales follow

    if (warp == 0) {
        // ---------------- producer ----------------
        if (lane == 0) {
            uint32_t it = 0, n_items_seen = 0;
            int cur_item = -1;
            bool live = true;
            const uint64_t pol = l2_policy_evict_first();
            // the slot of a work item is read once per item, and the next item's one tile ahead: a global load in front of
            // every tile's first copy is a bubble the ring (a few microseconds of stages) does not always hide
            int slot = tile_lo < tile_hi ? a.item_slot[(int)(tile_lo / RB)] : 0, next_slot = slot;
            for (long tile = tile_lo; tile < tile_hi && live; ++tile) {
                const int item = (int)(tile / RB), rb = (int)(tile % RB);
                if (item != cur_item) {  // new work item: its activation image replaces the previous one
                    if (cur_item >= 0) slot = next_slot;
                    if (!mbar_wait(smem_u32(b_empty), (n_items_seen & 1u) ^ 1u)) { atomicOr(a.counters + 2, kStatusFp4Timeout); break; }
                    mbar_expect_tx(smem_u32(b_full), (uint32_t)NS * kF4BStage);
                    bulk_g2s(smem_u32(bimg), a.bq + (size_t)item * NS * kF4BStage, (uint32_t)NS * kF4BStage, smem_u32(b_full));
                    cur_item = item;
                    ++n_items_seen;
                    if ((long)(item + 1) * RB < tile_hi) next_slot = a.item_slot[item + 1];  // in flight while this item streams
                }
                const uint8_t* asrc = (slot >= a.n_slots ? a.sh_bank_t : a.bank_t + (size_t)slot * RB * NS * kF4AStage) +
                                      (size_t)rb * NS * kF4AStage;
                const int sb = st_begin(tile), se = st_end(tile);
                for (int st = sb; st < se; ++st, ++it) {
                    const int s = (int)(it % (uint32_t)S);
                    if (!mbar_wait(smem_u32(&empty[s]), ((it / (uint32_t)S) & 1u) ^ 1u)) {
                        atomicOr(a.counters + 2, kStatusFp4Timeout);
                        live = false;
                        break;
                    }
                    mbar_expect_tx(smem_u32(&full[s]), kF4AStage);
                    bulk_g2s_stream(smem_u32(stages + (size_t)s * kF4AStage), asrc + (size_t)st * kF4AStage, kF4AStage, smem_u32(&full[s]), pol);
                }
            }
            // drain: copies handed to the copy engine must land before the CTA may exit
            for (uint32_t back = 0; back < (uint32_t)S && back < it; ++back) {
                const uint32_t j = it - 1 - back;
                if (!mbar_wait(smem_u32(&full[j % (uint32_t)S]), (j / (uint32_t)S) & 1u)) { atomicOr(a.counters + 2, kStatusFp4Timeout); break; }
            }
            if (n_items_seen > 0 && !mbar_wait(smem_u32(b_full), (n_items_seen - 1) & 1u)) atomicOr(a.counters + 2, kStatusFp4Timeout);
        }
    } else if (warp == 1 || warp == 6) {
        // ---------------- MMA issuers ----------------
        // Issuer A (warp 1) takes the even stages of every tile, issuer B (warp 6) the odd ones; each owns an
        // accumulator per buffer and the epilogue adds the two. Scale blocks travel to tensor memory with tcgen05.cp:
        // the bank scales of an issuer's next stage are copied before the MMAs of its current stage are issued (when
        // that stage has already landed), the activation scales of a work item once per item (each issuer its stages).
        const uint32_t me = warp == 1 ? 0u : 1u;
        if (lane == 0 && me < n_issuers) {
            const uint32_t idesc = idesc_nvf4(kF4ARows, kF4BRows);
            const uint32_t tmem_sfb_item = tmem_sf0 + S * 16;  // NS x 16 columns when resident
            // descriptor words: smem address >> 4 in the low 14 bits; LBO >> 4 at bit 16; SBO = 128 B, version 1 in the high word
            const uint32_t hi_word = 0x00004008u;
            const uint32_t a_lo0 = ((smem_u32(stages) >> 4) & 0x3FFFu) | ((uint32_t)(kF4ARows * 16 >> 4) << 16);
            const uint32_t b_lo0 = ((smem_u32(bimg) >> 4) & 0x3FFFu) | ((uint32_t)(kF4BRows * 16 >> 4) << 16);
            const uint32_t sfa_lo0 = (smem_u32(stages + kF4ANib) >> 4) & 0x3FFFu;
            const uint32_t sfb_lo0 = (smem_u32(bimg + kF4BNib) >> 4) & 0x3FFFu;
            uint32_t tcount = 0, n_items_seen = 0;
            uint32_t sfa_done = 0;  // this issuer's stages below sfa_done have their bank scales in tensor memory
            int cur_item = -1;
            bool live = true;
            uint32_t it0 = 0;       // index of the tile's first stage in the CTA's stage sequence
            for (long tile = tile_lo; tile < tile_hi && live; ++tile, ++tcount) {
                const int item = (int)(tile / RB);
                const int sb = st_begin(tile), se = st_end(tile);
                if (item != cur_item) {
                    if (!mbar_wait(smem_u32(b_full), n_items_seen & 1u)) { atomicOr(a.counters + 2, kStatusFp4Timeout); break; }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    if (sfb_resident)
                        for (int st = 0; st < NS; ++st)
                            if (((uint32_t)st & (n_issuers - 1u)) == me)  // the stages this issuer will multiply
#pragma unroll
                                for (int j = 0; j < 4; ++j)
                                    tc_cp_sf_lo(tmem_sfb_item + 16 * st + 4 * j, sfb_lo0 + (uint32_t)((st * kF4BStage + 512 * j) >> 4));
                    cur_item = item;
                    ++n_items_seen;
                }
                const bool last_of_item = (tile + 1 >= tile_hi) || ((int)((tile + 1) / RB) != item);
                const uint32_t buf = tcount & 1u;
                if (!mbar_wait(smem_u32(&acc_empty[buf]), ((tcount >> 1) & 1u) ^ 1u)) { atomicOr(a.counters + 2, kStatusFp4Timeout); break; }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t tmem_d = tmem + buf * 64 + me * 32;
                bool first = true;
                for (int st = sb; st < se; ++st) {
                    const uint32_t it = it0 + (uint32_t)(st - sb);
                    if (((uint32_t)st & (n_issuers - 1u)) != me) continue;
                    const uint32_t s = it % (uint32_t)S, ph = (it / (uint32_t)S) & 1u;
                    if (sfa_done <= it) {  // not copied ahead: wait for the stage and copy now
                        if (!mbar_wait(smem_u32(&full[s]), ph)) { atomicOr(a.counters + 2, kStatusFp4Timeout); live = false; break; }
                        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                        const uint32_t lo = sfa_lo0 + s * (kF4AStage >> 4);
#pragma unroll
                        for (int j = 0; j < 4; ++j) tc_cp_sf_lo(tmem_sf0 + s * 16 + 4 * j, lo + j * 32);
                        sfa_done = it + 1;
                    }
                    const uint32_t nx = it + n_issuers;  // this issuer's next stage, when it lies in the same tile
                    if (st + (int)n_issuers < se && sfa_done <= nx) {
                        const uint32_t sn = nx % (uint32_t)S, phn = (nx / (uint32_t)S) & 1u;
                        if (mbar_test(smem_u32(&full[sn]), phn)) {
                            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                            const uint32_t lo = sfa_lo0 + sn * (kF4AStage >> 4);
#pragma unroll
                            for (int j = 0; j < 4; ++j) tc_cp_sf_lo(tmem_sf0 + sn * 16 + 4 * j, lo + j * 32);
                            sfa_done = nx + 1;
                        }
                    }
                    const uint32_t a_lo = a_lo0 + s * (kF4AStage >> 4), b_lo = b_lo0 + (uint32_t)st * (kF4BStage >> 4);
                    const uint32_t sfa = tmem_sf0 + s * 16;
                    uint32_t sfb = tmem_sfb_item + st * 16;
                    if (!sfb_resident) {
                        sfb = tmem_sf0 + S * 16 + (s & 3) * 16;  // 4 small slots: consecutive stages of either issuer never collide
#pragma unroll
                        for (int j = 0; j < 4; ++j) tc_cp_sf_lo(sfb + 4 * j, sfb_lo0 + (uint32_t)((st * kF4BStage + 512 * j) >> 4));
                    }
                    if (first) tc_mma_nvf4_lo<false>(tmem_d, a_lo, hi_word, b_lo, hi_word, idesc, sfa, sfb);
                    else tc_mma_nvf4_lo<true>(tmem_d, a_lo, hi_word, b_lo, hi_word, idesc, sfa, sfb);
                    first = false;
#pragma unroll
                    for (int j = 1; j < 4; ++j)
                        tc_mma_nvf4_lo<true>(tmem_d, a_lo + j * (2 * kF4ARows * 16 >> 4), hi_word, b_lo + j * (2 * kF4BRows * 16 >> 4), hi_word,
                                             idesc, sfa + 4 * j, sfb + 4 * j);
                    tc_commit_f4(smem_u32(&empty[s]));
                }
                if (live) {
                    tc_commit_f4(smem_u32(&acc_full[buf]));
                    if (last_of_item) tc_commit_f4(smem_u32(b_empty));  // every MMA of this issuer that reads the activation image is done
                }
                it0 += (uint32_t)(se - sb);
            }
        }
    } else if (warp < 6) {
        // ---------------- epilogue warps (TMEM lane quarter = warp % 4) ----------------
        // Thread = bank row (quarter * 32 + lane) for all pairs of the item. The 128-point Walsh-Hadamard transform over
        // the rows runs where the rows are: five butterfly stages across the lanes (shuffles), the two stages across the
        // lane quarters through one shared-memory exchange - one barrier per tile, all four warps busy however few
        // pairs the item holds.
        const int quarter = warp & 3, et = tid - 64;
        const int row = quarter * 32 + lane;
        const bool q0 = (quarter & 1) != 0, q1 = (quarter & 2) != 0;
        uint32_t tcount = 0, zpar = 0;
        // per work item (the tiles of an item follow one another): its pairs, their scales and experts. Fetched when the
        // item changes, not per tile - the chain item -> pairs -> experts -> sign words is several memory round trips,
        // longer than a short tile streams
        int cur_item = -1, start = 0, cnt = 0;
        bool sh = false;
        float s2_lo = 0.0f, s2_hi = 0.0f, ps8[8];
        int ex8[8];
        for (long tile = tile_lo; tile < tile_hi; ++tile, ++tcount) {
            const int item = (int)(tile / RB), rb = (int)(tile % RB);
            if (item != cur_item) {
                cur_item = item;
                start = a.item_start[item];
                cnt = a.item_cnt[item];
                const int slot = a.item_slot[item];
                sh = slot >= a.n_slots;
                s2_lo = sh ? a.sh_s2[0] : a.s2[slot];
                s2_hi = sh ? a.sh_s2[a.sh_split < R ? 1 : 0] : s2_lo;
#pragma unroll
                for (int n = 0; n < 8; ++n) {
                    ps8[n] = n < cnt ? a.pscale[start + n] : 0.0f;
                    ex8[n] = (n < cnt && !sh) ? a.pair_expert[start + n] : 0;
                }
            }
            // a partial tile (a slice of the contraction): which issuers multiplied anything, and the result is added
            const int sb = st_begin(tile), se = st_end(tile);
            const bool partial = sb > 0 || se < NS;
            const bool has_a = n_issuers == 1 || sb + (sb & 1) < se, has_b = n_issuers == 2 && sb + ((sb & 1) ^ 1) < se;
            // operands of the epilogue that depend on the row block, fetched while the tile streams
            const float s2 = rb * 128 >= a.sh_split ? s2_hi : s2_lo;
            float g8[8];
            uint32_t sbits = 0u;  // bit n: r_s2 sign of this thread's row for pair n
#pragma unroll
            for (int n = 0; n < 8; ++n) {
                g8[n] = ps8[n] * s2;
                if (n < cnt && !sh) sbits |= ((a.rs2[(size_t)ex8[n] * (R / 32) + rb * 4 + quarter] >> lane) & 1u) << n;
            }
            const uint32_t buf = tcount & 1u;
            // the 128 epilogue threads must take the same branch: a named barrier ORs their verdicts
            uint32_t fail = mbar_wait(smem_u32(&acc_full[buf]), (tcount >> 1) & 1u) ? 0u : 1u;
            asm volatile("{\n.reg .pred p, q;\nsetp.ne.u32 q, %1, 0;\nbarrier.red.or.pred p, 2, 128, q;\nselp.u32 %0, 1, 0, p;\n}"
                         : "=r"(fail) : "r"(fail) : "memory");
            if (fail) { if (et == 0) atomicOr(a.counters + 2, kStatusFp4Timeout); break; }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            uint32_t d[32];
            if (has_a) {
                tmem_ld32_f4(tmem + buf * 64 + ((uint32_t)(quarter * 32) << 16), d);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            } else {
#pragma unroll
                for (int n = 0; n < 32; ++n) d[n] = 0u;
            }
            if (has_b) {  // add issuer B's accumulator
                uint32_t d2[32];
                tmem_ld32_f4(tmem + buf * 64 + 32 + ((uint32_t)(quarter * 32) << 16), d2);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int n = 0; n < 24; ++n) d[n] = __float_as_uint(__uint_as_float(d[n]) + __uint_as_float(d2[n]));
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&acc_empty[buf]));  // accumulator buffer may be overwritten
            float v8[8];
#pragma unroll
            for (int n = 0; n < 8; ++n) {
                float v = (__uint_as_float(d[n]) + 0.03125f * __uint_as_float(d[8 + n]) + 0.0009765625f * __uint_as_float(d[16 + n])) * g8[n];
                v8[n] = ((sbits >> n) & 1u) ? -v : v;
            }
            float* zrow = a.zout + (size_t)start * R + rb * 128 + row;
            if (sh) {  // plain weights: no sign, no transform
#pragma unroll
                for (int n = 0; n < 8; ++n)
                    if (n < cnt) {
                        if (partial) atomicAdd(&zrow[(size_t)n * R], v8[n]);
                        else zrow[(size_t)n * R] = v8[n];
                    }
                continue;
            }
            float(*z)[128] = zs[zpar & 1u];
            ++zpar;
#pragma unroll
            for (int n = 0; n < 8; ++n) {
                if (n < cnt) {  // cnt is uniform over the warp
                    float v = v8[n];
#pragma unroll
                    for (int m = 1; m < 32; m <<= 1) {
                        const float o = __shfl_xor_sync(0xffffffffu, v, m);
                        v = (lane & m) ? (o - v) : (v + o);
                    }
                    z[n][row] = v;
                }
            }
            asm volatile("bar.sync 2, 128;" ::: "memory");
#pragma unroll
            for (int n = 0; n < 8; ++n) {
                if (n < cnt) {
                    const float a0 = z[n][lane], a1 = z[n][32 + lane], a2 = z[n][64 + lane], a3 = z[n][96 + lane];
                    const float lo = a0 + (q0 ? -a1 : a1), hi = a2 + (q0 ? -a3 : a3);
                    const float out = (lo + (q1 ? -hi : hi)) * 0.08838834764831845f;
                    if (partial) atomicAdd(&zrow[(size_t)n * R], out);  // the transform is linear: the two slices of a tile just add
                    else zrow[(size_t)n * R] = out;
                }
            }
            // no second barrier: the next tile writes the other buffer, and nobody reaches the tile after it before every
            // thread has passed the next tile's barrier
        }
    } else if (SIDE) {
        // ---------------- side warps: the healer product of this pass, chunk by chunk ----------------
        const int sw = warp - 7;
        switch (a.side.rank / 16) {
            case 1: side_healer<1>(a, hsm, sw, lane); break;
            case 2: side_healer<2>(a, hsm, sw, lane); break;
            case 4: side_healer<4>(a, hsm, sw, lane); break;
            default: side_healer<8>(a, hsm, sw, lane); break;
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kF4TmemCols) : "memory");
}

static int launch_bank_fp4_impl(const chronos_layer_t& L, int stage, const Plan& p, bool side, const void* x, int x_dtype, cudaStream_t st) {
    Fp4Args a{};
    a.K = stage == 0 ? L.hidden : L.inter;
    a.R = stage == 0 ? 2 * L.inter : L.hidden;
    a.bank_t = stage == 0 ? L.gu_t : L.dn_t;
    a.sh_bank_t = stage == 0 ? L.sh_gu_t : L.sh_dn_t;
    a.s2 = stage == 0 ? L.gu_s2 : L.dn_s2;
    a.sh_s2 = stage == 0 ? L.sh_gu_s2 : L.sh_dn_s2;
    a.sh_split = stage == 0 ? L.inter : 0x7fffffff;
    a.rs2 = stage == 0 ? L.gu_rs2 : L.dn_rs2;
    a.bq = stage == 0 ? p.bq_gu : p.bq_dn;
    a.pscale = stage == 0 ? p.pscale_gu : p.pscale_dn;
    a.zout = stage == 0 ? p.z1 : p.y1;
    a.item_start = p.item_start;
    a.item_cnt = p.item_cnt;
    a.item_slot = p.item_slot;
    a.pair_expert = p.pair_expert;
    a.counters = p.counters;
    a.n_slots = L.n_slots;
    a.split_tiles = side ? 1 : 0;  // the fused decode path zero-initialises z1 / y1 (front and mid kernels)
    if (side) {
        Fp4Side& sd = a.side;
        sd.kind = stage == 0 ? 1 : 2;
        sd.u = stage == 0 ? L.u_gu : L.u_dn;
        sd.v = stage == 0 ? L.v_gu : L.v_dn;
        sd.x = x;
        sd.x_dtype = x_dtype;
        sd.pair_token = p.pair_token;
        sd.ac = p.ac;
        sd.pscale = stage == 0 ? p.pscale_gu : p.pscale_dn;
        sd.heal = stage == 0 ? p.heal_gu : p.heal_dn;
        sd.chunk_start = p.gitem_start;
        sd.chunk_cnt = p.gitem_cnt;
        sd.rank = L.rank;
        sd.n_experts = L.n_experts;
        sd.kc = stage == 0 ? L.hidden : L.inter;
    }
    const int ns = a.K / kF4StageK;
    const size_t bimg = (size_t)ns * kF4BStage;
    const size_t budget = 214 * 1024;  // dynamic part; the kernel's static shared memory (barriers, exchange buffers) takes the rest
    if (bimg + 2 * (size_t)kF4AStage + 1024 > budget) {
        set_error("bank_fp4: K = %d columns need a %zu-byte activation image, too large for shared memory", a.K, bimg);
        return CHRONOS_E_SHAPE;
    }
    int stages = (int)((budget - 1024 - bimg) / kF4AStage);
    a.n_stages = stages > kF4MaxStages ? kF4MaxStages : stages;
    const size_t smem = bimg + (size_t)a.n_stages * kF4AStage + 1024;
    const void* fn = side ? reinterpret_cast<const void*>(bank_fp4_kernel<true>) : reinterpret_cast<const void*>(bank_fp4_kernel<false>);
    if (int rc = ensure_dynamic_smem(fn, smem, "bank_fp4")) return rc;
    const int grid = bank_fp4_grid(L, stage, p);
    if (side) bank_fp4_kernel<true><<<grid, kF4Threads + kF4SideThreads, smem, st>>>(a);
    else bank_fp4_kernel<false><<<grid, kF4Threads, smem, st>>>(a);
    return check_launch("bank_fp4");
}

int launch_bank_fp4(const chronos_layer_t& L, int stage, const Plan& p, cudaStream_t st) { return launch_bank_fp4_impl(L, stage, p, false, nullptr, 0, st); }
int launch_bank_fp4_fused(const chronos_layer_t& L, int stage, const Plan& p, const void* x, int x_dtype, cudaStream_t st) {
    return launch_bank_fp4_impl(L, stage, p, true, x, x_dtype, st);
}

// ---------------------------------------------------------------------------------------------------------------
// FP4 tensor regime (large batches): the same block-scaled MMA with both operands streamed.
// Work item = up to 64 sorted pairs of ONE expert; its activation image per 256-column stage holds 192 rows
// (row = term * 64 + position): 24576 B of nibbles, byte(r, c, b) at c * 3072 + r * 16 + b, then per MMA two 512-byte
// scale blocks (rows 0-127, rows 128-191). Tile = (work item, 128 bank rows): D[128 x 192] in tensor memory, two
// buffers, so the epilogue of a tile overlaps the MMAs of the next.
// 10 warps: producer (per stage one 18432 B bank copy + one 28672 B activation copy into a 4-deep ring), MMA issuer
// (per stage 12 scale-block copies to tensor memory + 4 MMAs of 128 x 192 x 64), 8 epilogue warps (TMEM lane quarter =
// warp % 4; warps 2-5 take positions 0-31, warps 6-9 positions 32-63): sum the 3 terms, transpose through shared
// memory, then per pair scale, r_s2 sign, FWHT128 over the bank rows, store.
// ---------------------------------------------------------------------------------------------------------------
constexpr int kWStages = 4;
constexpr int kWStage = kF4AStage + kWideStageBytes;  // 47104
constexpr int kWThreads = 320;
constexpr int kWZsFloats = 2 * 32 * 132;

struct Fp4WideArgs {
    const uint8_t* bank_t; const uint8_t* sh_bank_t;
    const float* s2; const float* sh_s2; int sh_split;
    const uint32_t* rs2;
    const uint8_t* bq;         // [gitems, NS, 28672]
    const float* pscale;
    float* zout;               // [P, R]
    const int32_t* item_start; const int32_t* item_cnt; const int32_t* item_slot; const int32_t* pair_expert;
    int32_t* counters;
    int R, K, n_slots;
    // fused healer (NULL / 0 without it): per (expert, 128-row block) a K-major fp16 tile [rank/8][128][8] of the healer's
    // output factor in the basis of the accumulators, per work item a tile [rank/8][64][8] of its input factors
    const __half* ut; const __half* himg; int rank;
};

// kind::f16 instruction descriptor: D fp32 (bits 4-5 = 1), A = B = fp16 (format 0), K-major, N at [17,23), M at [24,29)
__device__ __forceinline__ uint32_t idesc_f16(int m, int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
// D[128 x N] += A[128 x 16] B[N x 16]^T, fp16 operands from shared memory, accumulating into the same tensor-memory
// columns the block-scaled MMAs of the tile wrote
__device__ __forceinline__ void tc_mma_f16_acc(uint32_t tmem_d, uint32_t da_lo, uint32_t da_hi, uint32_t db_lo, uint32_t db_hi,
                                               uint32_t idesc) {
    asm volatile(
        "{\n.reg .b64 a, b;\n.reg .pred p;\nmov.b64 a, {%1, %2};\nmov.b64 b, {%3, %4};\nsetp.eq.u32 p, 0, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %5, p;\n}" ::"r"(tmem_d),
        "r"(da_lo), "r"(da_hi), "r"(db_lo), "r"(db_hi), "r"(idesc)
        : "memory");
}


// NT = bank row blocks multiplied against one activation stage: 1 (two accumulator buffers, the epilogue overlaps the next
// tile) or 2 (more MMA work per staged byte: stage = 2 x 18432 + 28672 B, 3 stages, accumulators of the two row blocks side
// by side in tensor memory, single-buffered).
template <int NT>
__global__ void __launch_bounds__(kWThreads, 1) bank_fp4_wide_kernel(const Fp4WideArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t bars[2 * kWStages + 4];  // full[S], empty[S], acc_full[2], acc_empty[2]
    __shared__ uint32_t tmem_base_s;
    uint8_t* stages = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    constexpr int STG = NT == 2 ? 3 : kWStages;
    constexpr int STAGE = NT * kF4AStage + kWideStageBytes;
    constexpr uint32_t SFW = NT == 2 ? 16u : 12u;  // scale columns per MMA step: 4 per bank row block + 8 for the 192 activation rows
    float* zs = reinterpret_cast<float*>(stages + (size_t)STG * STAGE);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int R = a.R, RB = R / 128, NS = a.K / kF4StageK;
    constexpr uint32_t S = STG;
    const int RBT = RB / NT;  // tiles (groups of NT row blocks) per work item
    const long n_tiles = (long)a.counters[3] * RBT;
    // tiles go round-robin over the CTAs: at any moment the CTAs work on neighbouring tiles, i.e. on the same few work items
    // (whose activation image they share through L2) and on neighbouring row blocks of the same few banks
    const long tile_lo = blockIdx.x, tile_hi = n_tiles, tile_step = gridDim.x;
    // fused healer: work items before counters[4] belong to routed experts (the shared expert's items come last and have none)
    const int first_plain = a.ut != nullptr ? a.counters[4] : 0;
    const uint32_t ut_bytes = 128u * (uint32_t)a.rank * 2u, h_bytes = (uint32_t)kPairsPerWideItem * (uint32_t)a.rank * 2u;
    uint64_t* full = bars;
    uint64_t* empty = bars + kWStages;
    uint64_t* acc_full = bars + 2 * kWStages;
    uint64_t* acc_empty = bars + 2 * kWStages + 2;

    if (tid == 0) {
        for (int s = 0; s < STG; ++s) { mbar_init(smem_u32(&full[s]), 1); mbar_init(smem_u32(&empty[s]), 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(smem_u32(&acc_full[b]), 1); mbar_init(smem_u32(&acc_empty[b]), 8); }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)), "r"(512u) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base_s;  // columns: D buffer 0 at 0, D buffer 1 at 192, scale slots from 384

    if (warp == 0) {
        // ---------------- producer ----------------
        if (lane == 0) {
            uint32_t it = 0;
            bool live = true;
            for (long tile = tile_lo; tile < tile_hi && live; tile += tile_step) {
                const int item = (int)(tile / RBT), rb = (int)(tile % RBT) * NT;
                const int slot = a.item_slot[item];
                const uint8_t* asrc = (slot >= a.n_slots ? a.sh_bank_t : a.bank_t + (size_t)slot * RB * NS * kF4AStage) +
                                      (size_t)rb * NS * kF4AStage;
                const uint8_t* bsrc = a.bq + (size_t)item * NS * kWideStageBytes;
                for (int st = 0; st < NS; ++st, ++it) {
                    const uint32_t s = it % S;
                    if (!mbar_wait(smem_u32(&empty[s]), ((it / S) & 1u) ^ 1u)) {
                        atomicOr(a.counters + 2, kStatusFp4Timeout);
                        live = false;
                        break;
                    }
                    uint8_t* dst = stages + (size_t)s * STAGE;
                    mbar_expect_tx(smem_u32(&full[s]), STAGE);
#pragma unroll
                    for (int d = 0; d < NT; ++d)  // row block rb + d of the same slot: NS stages further on in the bank image
                        bulk_g2s(smem_u32(dst + d * kF4AStage), asrc + ((size_t)d * NS + st) * kF4AStage, kF4AStage, smem_u32(&full[s]));
                    bulk_g2s(smem_u32(dst + NT * kF4AStage), bsrc + (size_t)st * kWideStageBytes, kWideStageBytes, smem_u32(&full[s]));
                }
                if (live && item < first_plain) {  // one more ring slot: the healer tiles of the row blocks and the item's factors
                    const uint32_t s = it % S;
                    if (!mbar_wait(smem_u32(&empty[s]), ((it / S) & 1u) ^ 1u)) {
                        atomicOr(a.counters + 2, kStatusFp4Timeout);
                        break;
                    }
                    uint8_t* dst = stages + (size_t)s * STAGE;
                    const int e = a.pair_expert[a.item_start[item]];
                    mbar_expect_tx(smem_u32(&full[s]), NT * ut_bytes + h_bytes);
#pragma unroll
                    for (int d = 0; d < NT; ++d)
                        bulk_g2s(smem_u32(dst + d * ut_bytes), a.ut + ((size_t)e * RB + rb + d) * (ut_bytes / 2), ut_bytes, smem_u32(&full[s]));
                    bulk_g2s(smem_u32(dst + NT * ut_bytes), a.himg + (size_t)item * (h_bytes / 2), h_bytes, smem_u32(&full[s]));
                    ++it;
                }
            }
            for (uint32_t back = 0; back < S && back < it; ++back) {  // copies in flight must land before the CTA exits
                const uint32_t j = it - 1 - back;
                if (!mbar_wait(smem_u32(&full[j % S]), (j / S) & 1u)) { atomicOr(a.counters + 2, kStatusFp4Timeout); break; }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = idesc_nvf4(kF4ARows, kWideRows);
            const uint32_t idesc_heal = idesc_f16(kF4ARows, kPairsPerWideItem);
            const uint32_t hi_word = 0x00004008u;
            const uint32_t a_lo0 = ((smem_u32(stages) >> 4) & 0x3FFFu) | ((uint32_t)(kF4ARows * 16 >> 4) << 16);
            const uint32_t b_lo0 = ((smem_u32(stages + NT * kF4AStage) >> 4) & 0x3FFFu) | ((uint32_t)(kWideRows * 16 >> 4) << 16);
            const uint32_t sfa_lo0 = (smem_u32(stages + kF4ANib) >> 4) & 0x3FFFu;
            const uint32_t sfb_lo0 = (smem_u32(stages + NT * kF4AStage + kWideRows * 128) >> 4) & 0x3FFFu;
            uint32_t it = 0, tcount = 0;
            bool live = true;
            for (long tile = tile_lo; tile < tile_hi && live; tile += tile_step, ++tcount) {
                const uint32_t buf = NT == 2 ? 0u : (tcount & 1u);
                const uint32_t eph = NT == 2 ? (tcount & 1u) : ((tcount >> 1) & 1u);
                if (!mbar_wait(smem_u32(&acc_empty[buf]), eph ^ 1u)) { atomicOr(a.counters + 2, kStatusFp4Timeout); break; }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t tmem_d = tmem + buf * kWideRows;
                for (int st = 0; st < NS; ++st, ++it) {
                    const uint32_t s = it % S;
                    if (!mbar_wait(smem_u32(&full[s]), (it / S) & 1u)) { atomicOr(a.counters + 2, kStatusFp4Timeout); live = false; break; }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    // scale blocks of the stage: per MMA 4 columns for the bank rows, 8 for the 192 activation rows; two
                    // sets of slots alternate between consecutive stages
                    const uint32_t sf = tmem + 2 * kWideRows + (it & 1u) * (4u * SFW);
                    const uint32_t so = s * (STAGE >> 4);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
#pragma unroll
                        for (int d = 0; d < NT; ++d) tc_cp_sf_lo(sf + SFW * j + 4 * d, sfa_lo0 + so + d * (kF4AStage >> 4) + j * 32);
                        tc_cp_sf_lo(sf + SFW * j + 4 * NT, sfb_lo0 + so + j * 64);
                        tc_cp_sf_lo(sf + SFW * j + 4 * NT + 4, sfb_lo0 + so + j * 64 + 32);
                    }
                    const uint32_t a_lo = a_lo0 + so, b_lo = b_lo0 + so;
#pragma unroll
                    for (int d = 0; d < NT; ++d) {  // row block d: its own bank tile, scales and accumulator, the same activations
                        const uint32_t ad = a_lo + d * (kF4AStage >> 4), dd = tmem_d + d * kWideRows;
                        if (st == 0) tc_mma_nvf4_lo<false>(dd, ad, hi_word, b_lo, hi_word, idesc, sf + 4 * d, sf + 4 * NT);
                        else tc_mma_nvf4_lo<true>(dd, ad, hi_word, b_lo, hi_word, idesc, sf + 4 * d, sf + 4 * NT);
#pragma unroll
                        for (int j = 1; j < 4; ++j)
                            tc_mma_nvf4_lo<true>(dd, ad + j * (2 * kF4ARows * 16 >> 4), hi_word, b_lo + j * (2 * kWideRows * 16 >> 4), hi_word,
                                                 idesc, sf + SFW * j + 4 * d, sf + SFW * j + 4 * NT);
                    }
                    tc_commit_f4(smem_u32(&empty[s]));
                }
                if (live && (int)(tile / RBT) < first_plain) {  // the healer step: rank / 16 MMAs of K = 16 per row block, N = 64
                    const uint32_t s = it % S;
                    if (!mbar_wait(smem_u32(&full[s]), (it / S) & 1u)) { atomicOr(a.counters + 2, kStatusFp4Timeout); break; }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t so = s * (STAGE >> 4);
                    const uint32_t u_lo = a_lo0 + so;  // same leading-dimension offset as the bank tile: 128 rows x 16 bytes
                    const uint32_t h_lo = (((smem_u32(stages) + NT * ut_bytes) >> 4) & 0x3FFFu) + so + ((uint32_t)(kPairsPerWideItem * 16 >> 4) << 16);
#pragma unroll
                    for (int d = 0; d < NT; ++d)
                        for (int kk = 0; kk < a.rank / 16; ++kk)
                            tc_mma_f16_acc(tmem_d + d * kWideRows, u_lo + d * (ut_bytes >> 4) + kk * (2 * kF4ARows * 16 >> 4), hi_word,
                                           h_lo + kk * (2 * kPairsPerWideItem * 16 >> 4), hi_word, idesc_heal);
                    tc_commit_f4(smem_u32(&empty[s]));
                    ++it;
                }
                if (live) tc_commit_f4(smem_u32(&acc_full[buf]));
            }
        }
    } else {
        // ---------------- epilogue warps ----------------
        const int ew = warp - 2, quarter = warp & 3, half = ew >> 2, wq = ew & 3;
        const int row = quarter * 32 + lane;
        float* zsh = zs + (size_t)half * 32 * 132;
        const int bar_id = 2 + half;
        uint32_t tcount = 0;
        for (long tile = tile_lo; tile < tile_hi; tile += tile_step, ++tcount) {
            const int item = (int)(tile / RBT), rb0 = (int)(tile % RBT) * NT;
            const int start = a.item_start[item], cnt = a.item_cnt[item], slot = a.item_slot[item];
            const bool sh = slot >= a.n_slots;
            const uint32_t buf = NT == 2 ? 0u : (tcount & 1u);
            const uint32_t fph = NT == 2 ? (tcount & 1u) : ((tcount >> 1) & 1u);
            uint32_t fail = mbar_wait(smem_u32(&acc_full[buf]), fph) ? 0u : 1u;
            asm volatile("{\n.reg .pred p, q;\nsetp.ne.u32 q, %1, 0;\nbarrier.red.or.pred p, %2, 128, q;\nselp.u32 %0, 1, 0, p;\n}"
                         : "=r"(fail) : "r"(fail), "r"(bar_id) : "memory");
            if (fail) { if (lane == 0 && wq == 0) atomicOr(a.counters + 2, kStatusFp4Timeout); break; }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int n0 = half * 32;
#pragma unroll
            for (int d = 0; d < NT; ++d) {
                const int rb = rb0 + d;
                const float s2 = sh ? a.sh_s2[rb * 128 >= a.sh_split ? 1 : 0] : a.s2[slot];
                uint32_t sw = 0u;  // r_s2 sign bits of this lane's 4 rows (one expert per work item)
                if (!sh) sw = a.rs2[(size_t)a.pair_expert[start] * (R / 32) + rb * 4 + lane / 8] >> ((lane & 7) * 4);
                if (n0 < cnt) {
                    const uint32_t tbase = tmem + (buf + d) * kWideRows + (uint32_t)n0 + ((uint32_t)(quarter * 32) << 16);
#pragma unroll
                    for (int ch = 0; ch < 2; ++ch) {
                        uint32_t t0[16], t1[16], t2[16];
                        tmem_ld16_f4(tbase + ch * 16, t0);
                        tmem_ld16_f4(tbase + 64 + ch * 16, t1);
                        tmem_ld16_f4(tbase + 128 + ch * 16, t2);
                        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                        for (int n = 0; n < 16; ++n)
                            zsh[(ch * 16 + n) * 132 + row] =
                                __uint_as_float(t0[n]) + 0.03125f * __uint_as_float(t1[n]) + 0.0009765625f * __uint_as_float(t2[n]);
                    }
                }
                if (d == NT - 1) {  // every accumulator of the tile has been read: the issuer may overwrite them
                    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) mbar_arrive(smem_u32(&acc_empty[buf]));
                }
                asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
#pragma unroll 2
                for (int i = 0; i < 8; ++i) {
                    const int n = n0 + wq * 8 + i;
                    if (n < cnt) {
                        const float g = a.pscale[start + n] * s2;
                        const float4 t4 = *reinterpret_cast<const float4*>(&zsh[(wq * 8 + i) * 132 + lane * 4]);
                        float v[4] = {t4.x * g, t4.y * g, t4.z * g, t4.w * g};
                        if (!sh) {
#pragma unroll
                            for (int q = 0; q < 4; ++q)
                                if ((sw >> q) & 1u) v[q] = -v[q];
                            fwht128_warp(v, lane);
                        }
                        *reinterpret_cast<float4*>(a.zout + (size_t)(start + n) * R + rb * 128 + lane * 4) = make_float4(v[0], v[1], v[2], v[3]);
                    }
                }
                asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u) : "memory");
}

int launch_bank_fp4_wide(const chronos_layer_t& L, int stage, const Plan& p, cudaStream_t st) {
    Fp4WideArgs a{};
    a.K = stage == 0 ? L.hidden : L.inter;
    a.R = stage == 0 ? 2 * L.inter : L.hidden;
    a.bank_t = stage == 0 ? L.gu_t : L.dn_t;
    a.sh_bank_t = stage == 0 ? L.sh_gu_t : L.sh_dn_t;
    a.s2 = stage == 0 ? L.gu_s2 : L.dn_s2;
    a.sh_s2 = stage == 0 ? L.sh_gu_s2 : L.sh_dn_s2;
    a.sh_split = stage == 0 ? L.inter : 0x7fffffff;
    a.rs2 = stage == 0 ? L.gu_rs2 : L.dn_rs2;
    a.bq = stage == 0 ? p.bq_gu : p.bq_dn;
    a.pscale = stage == 0 ? p.pscale_gu : p.pscale_dn;
    a.zout = stage == 0 ? p.z1 : p.y1;
    a.item_start = p.gitem_start;
    a.item_cnt = p.gitem_cnt;
    a.item_slot = p.gitem_slot;
    a.pair_expert = p.pair_expert;
    a.counters = p.counters;
    a.n_slots = L.n_slots;
    if (healer_fused(L, p)) {
        a.ut = reinterpret_cast<const __half*>(stage == 0 ? L.ut_gu : L.ut_dn);
        a.himg = p.himg;
        a.rank = L.rank;
    }
    // the gate_up pass (16 stages per tile) multiplies two row blocks per activation stage; the down pass (6 stages per
    // tile) keeps one row block and the overlapped epilogue
    bool two = stage == 0 && (a.R / 128) % 2 == 0;
    size_t smem = (size_t)3 * (2 * kF4AStage + kWideStageBytes) + (size_t)kWZsFloats * 4 + 1024;
    // the two-row-block form needs every byte of shared memory an SM has: fall back to one row block when it is refused
    if (two && ensure_dynamic_smem(reinterpret_cast<const void*>(bank_fp4_wide_kernel<2>), smem, "bank_fp4_wide") != CHRONOS_OK) two = false;
    if (!two) {
        smem = (size_t)kWStages * kWStage + (size_t)kWZsFloats * 4 + 1024;
        if (int rc = ensure_dynamic_smem(reinterpret_cast<const void*>(bank_fp4_wide_kernel<1>), smem, "bank_fp4_wide")) return rc;
    }
    const int sms = device_sm_count();
    const long max_tiles = (long)p.max_gitems * (a.R / 128);
    const int grid = (int)(max_tiles < sms ? max_tiles : sms);
    if (two) bank_fp4_wide_kernel<2><<<grid, kWThreads, smem, st>>>(a);
    else bank_fp4_wide_kernel<1><<<grid, kWThreads, smem, st>>>(a);
    return check_launch("bank_fp4_wide");
}

int launch_fp4_probe(const uint8_t* a_img, const uint8_t* b_img, int n_stages, int b_rows, float* d_out, int32_t* status,
                     cudaStream_t st) {
    const size_t smem = kF4AStage + (size_t)b_rows * 128 + 2048 * ((b_rows + 127) / 128) + 1024;
    if (int rc = ensure_dynamic_smem(reinterpret_cast<const void*>(fp4_mma_probe_kernel), smem, "fp4_probe")) return rc;
    fp4_mma_probe_kernel<<<1, 128, smem, st>>>(a_img, b_img, n_stages, b_rows, d_out, status);
    return check_launch("fp4_probe");
}

}  // namespace chronos
