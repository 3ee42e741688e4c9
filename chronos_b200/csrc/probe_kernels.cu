// Parity probes: NVFP4 dequantisation (bit-exact) and weight-space reconstruction of one expert.
#include "common.cuh"

namespace chronos {

__constant__ float kE2M1Lut[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                                   -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

// One thread per packed byte: two outputs. value = fl32(lut * fl32(float(e4m3) * s2)): the operand order of
// unpack_nvfp4 (chronos_1t/converter/convert_glm53_flash_colab.py:88-89); __fmul_rn forbids FMA contraction.
__global__ void dequant_nvfp4_kernel(const uint8_t* __restrict__ packed, const uint8_t* __restrict__ scale,
                                     const float* __restrict__ s2p, float* __restrict__ out, int rows, int cols) {
    const size_t n = (size_t)rows * (cols / 2);
    const float s2 = *s2p;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t row = i / (cols / 2), cb = i % (cols / 2);
        const uint8_t b = packed[i];
        const float sc = __fmul_rn(e4m3_to_f32(scale[row * (cols / 16) + cb / 8]), s2);
        float2 o;
        o.x = __fmul_rn(kE2M1Lut[b & 15], sc);
        o.y = __fmul_rn(kE2M1Lut[b >> 4], sc);
        reinterpret_cast<float2*>(out)[i] = o;
    }
}

int launch_dequant(const uint8_t* packed, const uint8_t* scale, const float* s2, float* out, int rows, int cols,
                   cudaStream_t st) {
    const size_t n = (size_t)rows * (cols / 2);
    const int blocks = (int)((n + 255) / 256 < 148 * 16 ? (n + 255) / 256 : 148 * 16);
    dequant_nvfp4_kernel<<<blocks, 256, 0, st>>>(packed, scale, s2, out, rows, cols);
    return check_launch("dequant_nvfp4");
}

// Row-axis half of the unbind: scratch[rb*128 + :, j] = H_128( r_s2 * S[rb*128 + :, j] ).
// One warp per (128-row block, column): lane l holds rows 4l..4l+3.
__global__ void unfold_rows_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ s, const float* __restrict__ s2p,
                                   const uint32_t* __restrict__ rs2, float* __restrict__ scratch, int rows, int cols) {
    const int lane = threadIdx.x & 31;
    const float s2 = *s2p;
    const size_t warp = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
    const size_t total = (size_t)(rows / 128) * cols;
    if (warp >= total) return;
    const int rb = (int)(warp / cols), j = (int)(warp % cols);
    float v[4];
    const uint32_t sw = rs2[rb * 4 + lane / 8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int row = rb * 128 + lane * 4 + i;
        const uint8_t b = w[(size_t)row * (cols / 2) + j / 2];
        const float sc = __fmul_rn(e4m3_to_f32(s[(size_t)row * (cols / 16) + j / 16]), s2);
        float val = __fmul_rn(kE2M1Lut[(j & 1) ? (b >> 4) : (b & 15)], sc);
        if ((sw >> ((lane & 7) * 4 + i)) & 1u) val = -val;
        v[i] = val;
    }
    fwht128_warp(v, lane);
#pragma unroll
    for (int i = 0; i < 4; ++i) scratch[(size_t)(rb * 128 + lane * 4 + i) * cols + j] = v[i];
}

// Column-axis half + healer: out[i, c_perm[j']] = c_s1 * H_128( c_s2 * r_s1[i] * scratch[r_inv[i], :] )[j'] * beta
//                                               + sum_c U[i, c] V[c, .].  One warp per (output row, 128-column block).
__global__ void unfold_cols_kernel(const float* __restrict__ scratch, const uint16_t* __restrict__ rout,
                                   const uint16_t* __restrict__ cin, const uint32_t* __restrict__ cs2, const float* __restrict__ betap,
                                   const uint8_t* __restrict__ u, const uint8_t* __restrict__ vmat, int v_is_transposed,
                                   int rank, float* __restrict__ out, int rows, int cols) {
    const int lane = threadIdx.x & 31;
    const size_t warp = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
    const size_t total = (size_t)rows * (cols / 128);
    if (warp >= total) return;
    const float beta = *betap;
    const int i = (int)(warp / (cols / 128)), cb = (int)(warp % (cols / 128));
    const uint16_t ro = rout[i];
    const int src = ro & 0x7fff;
    const float rsign = (ro >> 15) ? -1.0f : 1.0f;
    const uint32_t sw = cs2[cb * 4 + lane / 8];
    float v[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int jp = cb * 128 + lane * 4 + q;
        float val = scratch[(size_t)src * cols + jp] * rsign;
        if ((sw >> ((lane & 7) * 4 + q)) & 1u) val = -val;
        v[q] = val;
    }
    fwht128_warp(v, lane);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int jp = cb * 128 + lane * 4 + q;
        const uint16_t ce = cin[jp];
        const int j = ce & 0x7fff;
        float val = (ce >> 15) ? -v[q] : v[q];
        float heal = 0.0f;
        for (int c = 0; c < rank; ++c) {
            const float uv = e4m3_to_f32(u[(size_t)i * rank + c]);
            const float vv = e4m3_to_f32(v_is_transposed ? vmat[(size_t)j * rank + c] : vmat[(size_t)c * cols + j]);
            heal = fmaf(uv, vv, heal);
        }
        out[(size_t)i * cols + j] = beta * val + heal;
    }
}

int launch_unfold(const chronos_layer_t& L, int expert, int which, float* out, float* scratch, cudaStream_t st) {
    const int rows = which == 0 ? 2 * L.inter : L.hidden, cols = which == 0 ? L.hidden : L.inter;
    const int slot = expert / L.group_size;
    const uint8_t* w = (which == 0 ? L.gu_w : L.dn_w) + (size_t)slot * rows * (cols / 2);
    const uint8_t* s = (which == 0 ? L.gu_s : L.dn_s) + (size_t)slot * rows * (cols / 16);
    const float* s2p = (which == 0 ? L.gu_s2 : L.dn_s2) + slot;
    const float* betap = (which == 0 ? L.gu_beta : L.dn_beta) + expert;
    // the two per-slot / per-expert scalars are read by the kernels through their device pointers: the probe is
    // stream-ordered like every other entry point (no copy to the host, no synchronisation)
    const uint32_t* rs2 = (which == 0 ? L.gu_rs2 : L.dn_rs2) + (size_t)expert * (rows / 32);
    const uint16_t* rout = (which == 0 ? L.gu_rout : L.dn_rout) + (size_t)expert * rows;
    const uint16_t* cin = (which == 0 ? L.gu_cin : L.dn_cin) + (size_t)expert * cols;
    const uint32_t* cs2 = (which == 0 ? L.gu_cs2 : L.dn_cs2) + (size_t)expert * (cols / 32);
    const uint8_t* u = (which == 0 ? L.u_gu : L.u_dn) + (size_t)expert * rows * L.rank;
    const uint8_t* v = (which == 0 ? L.v_gu : L.v_dn_t) + (size_t)expert * cols * L.rank;
    size_t warps = (size_t)(rows / 128) * cols;
    unfold_rows_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(w, s, s2p, rs2, scratch, rows, cols);
    if (int rc = check_launch("unfold_rows")) return rc;
    warps = (size_t)rows * (cols / 128);
    unfold_cols_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(scratch, rout, cin, cs2, betap, u, v, which == 1,
                                                                   L.rank, out, rows, cols);
    return check_launch("unfold_cols");
}

// ---------------------------------------------------------------------------------------------------------------
// Wait probe: exercises the give-up path every kernel of the library shares. One thread arms a shared-memory barrier
// for bytes that nobody ever sends, polls it through the same bounded wait the bank kernels use - with the caller's
// small poll limit - and, when the limit is reached, raises the status bit and returns normally. Nothing traps,
// nothing hangs, the context stays usable.
// ---------------------------------------------------------------------------------------------------------------
__global__ void wait_probe_kernel(int32_t* __restrict__ status, uint32_t poll_limit) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bar), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        mbar_expect_tx(smem_u32(&bar), 16);  // 16 bytes that no copy will deliver
        if (!mbar_wait(smem_u32(&bar), 0, poll_limit)) atomicOr(status, kStatusWaitProbeTimeout);
    }
}

int launch_wait_probe(int32_t* status, uint32_t poll_limit, cudaStream_t st) {
    wait_probe_kernel<<<1, 32, 0, st>>>(status, poll_limit);
    return check_launch("wait_probe");
}

// ---------------------------------------------------------------------------------------------------------------
// Allocation-free variant of the reconstruction probe: the row-axis intermediate lives in a fixed device array that
// is part of the library image, so the caller hands over nothing but the layer and the output.
// ---------------------------------------------------------------------------------------------------------------
constexpr size_t kStaticScratchFloats = size_t(4) << 20;  // 4 Mi floats = 16 MiB: matrices up to rows * cols = 4,194,304
static __device__ __align__(256) float g_unfold_scratch[kStaticScratchFloats];

constexpr int kMaxDevices = 64;
static float* g_unfold_scratch_addr[kMaxDevices];  // device address of the array on each device, filled at set-up

// Set-up for the CURRENT device (first call on that device only): the array's name is a host-side handle, not an
// address a kernel can use, so its device address is looked up once and cached.
static int static_scratch_for_current_device(float** out) {
    int dev = -1;
    cudaError_t rc = cudaGetDevice(&dev);
    if (rc != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        set_error("unfold_static: cannot identify the current device (%s)", rc == cudaSuccess ? "index out of range" : cudaGetErrorString(rc));
        return CHRONOS_E_LAUNCH;
    }
    if (g_unfold_scratch_addr[dev] == nullptr) {
        float* ptr = nullptr;
        rc = cudaGetSymbolAddress((void**)&ptr, g_unfold_scratch);
        if (rc != cudaSuccess || ptr == nullptr) {
            set_error("unfold_static: cudaGetSymbolAddress failed on device %d: %s", dev, cudaGetErrorString(rc));
            return CHRONOS_E_LAUNCH;
        }
        g_unfold_scratch_addr[dev] = ptr;
    }
    *out = g_unfold_scratch_addr[dev];
    return CHRONOS_OK;
}

int launch_unfold_static(const chronos_layer_t& L, int expert, int which, float* out, cudaStream_t st) {
    const size_t rows = which == 0 ? 2 * (size_t)L.inter : (size_t)L.hidden, cols = which == 0 ? (size_t)L.hidden : (size_t)L.inter;
    if (rows * cols > kStaticScratchFloats) {
        set_error("unfold_static: a %zu x %zu matrix needs %zu scratch floats, the built-in scratch holds %zu; "
                  "use chronos_b200_unfold_expert_fp32 with caller-provided scratch", rows, cols, rows * cols, kStaticScratchFloats);
        return CHRONOS_E_SHAPE;
    }
    float* scratch = nullptr;
    if (int rc = static_scratch_for_current_device(&scratch)) return rc;
    // every element of scratch[0 .. rows*cols) is written by the first kernel before the second reads it: no clearing needed
    return launch_unfold(L, expert, which, out, scratch, st);
}

}  // namespace chronos
