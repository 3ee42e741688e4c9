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

// instruction descriptor, block-scaled: A = B = e2m1 (code 1), K-major, scale format ue4m3 (0), N at [17,23), M at [24,29)
__device__ __forceinline__ uint32_t idesc_nvf4(int m, int n) {
    return (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// ---------------------------------------------------------------------------------------------------------------
// Operand-format probe: D[128, 32] = sum over n_stages * 256 columns of (A * scaleA) (B * scaleB)^T, one CTA.
// a_img: n_stages x 18432 B, b_img: n_stages x 6144 B in the layouts above. Used by the parity tests to pin the
// descriptor, scale-factor and nibble conventions against a plain dequantise-and-multiply on the CPU.
// ---------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(128, 1) fp4_mma_probe_kernel(const uint8_t* __restrict__ a_img,
                                                               const uint8_t* __restrict__ b_img, int n_stages,
                                                               float* __restrict__ d_out, int32_t* __restrict__ status) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t bars[2];  // stage landed, MMAs done
    __shared__ uint32_t tmem_base_s;
    uint8_t* sa = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* sb = sa + kF4AStage;  // 18432 is a multiple of 1024
    const int tid = threadIdx.x, warp = tid >> 5;
    if (tid == 0) {
        mbar_init(smem_u32(&bars[0]), 1);
        mbar_init(smem_u32(&bars[1]), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)), "r"(64u) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base_s;
    const uint32_t tmem_d = tmem, tmem_sfa = tmem + 32, tmem_sfb = tmem + 48;  // 32 + 16 + 16 columns
    const uint32_t idesc = idesc_nvf4(kF4ARows, kF4BRows);
    int failed = 0;
    for (int st = 0; st < n_stages && !failed; ++st) {
        if (tid == 0) {
            mbar_expect_tx(smem_u32(&bars[0]), kF4AStage + kF4BStage);
            bulk_g2s(smem_u32(sa), a_img + (size_t)st * kF4AStage, kF4AStage, smem_u32(&bars[0]));
            bulk_g2s(smem_u32(sb), b_img + (size_t)st * kF4BStage, kF4BStage, smem_u32(&bars[0]));
            bool ok = mbar_wait(smem_u32(&bars[0]), st & 1);
            if (ok) {
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    tc_cp_sf(tmem_sfa + 4 * j, smem_u32(sa + kF4ANib + 512 * j));
                    tc_cp_sf(tmem_sfb + 4 * j, smem_u32(sb + kF4BNib + 512 * j));
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint64_t da = smem_desc_interleaved(smem_u32(sa + 2 * j * (kF4ARows * 16)), kF4ARows * 16);
                    const uint64_t db = smem_desc_interleaved(smem_u32(sb + 2 * j * (kF4BRows * 16)), kF4BRows * 16);
                    tc_mma_nvf4(tmem_d, da, db, idesc, tmem_sfa + 4 * j, tmem_sfb + 4 * j, (st > 0 || j > 0) ? 1u : 0u);
                }
                tc_commit_f4(smem_u32(&bars[1]));
                ok = mbar_wait(smem_u32(&bars[1]), st & 1);  // single-buffered: wait before the next stage overwrites
            }
            if (!ok) atomicOr(status, 0x40);
        }
        failed = __syncthreads_or(tid == 0 ? (*(volatile int32_t*)status != 0) : 0);
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (!failed) {
        uint32_t r[32];
        tmem_ld32_f4(tmem_d + ((uint32_t)(warp * 32) << 16), r);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int i = 0; i < 32; ++i) d_out[(size_t)tid * 32 + i] = __uint_as_float(r[i]);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(64u) : "memory");
}

int launch_fp4_probe(const uint8_t* a_img, const uint8_t* b_img, int n_stages, float* d_out, int32_t* status,
                     cudaStream_t st) {
    const size_t smem = kF4AStage + kF4BStage + 1024;
    cudaError_t rc = cudaFuncSetAttribute(fp4_mma_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (rc != cudaSuccess) {
        set_error("fp4_probe: cannot opt in to %zu bytes of shared memory: %s", smem, cudaGetErrorString(rc));
        return CHRONOS_E_LAUNCH;
    }
    fp4_mma_probe_kernel<<<1, 128, smem, st>>>(a_img, b_img, n_stages, d_out, status);
    return check_launch("fp4_probe");
}

}  // namespace chronos
