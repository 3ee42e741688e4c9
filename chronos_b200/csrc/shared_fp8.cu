// Always-on shared expert kept in the stock 128 x 128 block-FP8 checkpoint format: float8_e4m3fn weights [N, K] with one
// fp32 `weight_scale_inv` per 128 x 128 block (chronos_1t/models/glm53_tiers.py:74-95 `dequant_fp8_block`; loaded and
// applied at chronos_1t/models/glm53_chronos_moe.py:170-181, :401-404: gate and up fused along the rows, then down).
//   y[t] += W_down . (silu(W_gate x[t]) * (W_up x[t]))           W = float(e4m3) * scale_inv[block]
// One GEMM kernel serves both products and every batch size: a CTA owns 128 weight rows (= one row of scale blocks) and
// 32 tokens; each warp multiplies its 16 rows, read straight from global memory once per token tile and converted
// e4m3 -> fp16 exactly, by the token tile staged in shared memory as fp16 (x / token scale), on mma.sync m16n8k16 with
// fp32 accumulation; the block scale is applied to the partial sum of every 128-column block in fp32 - the weights are
// never rounded to a 16-bit type, unlike the reference's dequantise-then-GEMM path. Decode-sized batches read the
// 18.9 MB of weights exactly once (HBM-bound); large batches re-read them from L2 once per 32 tokens.
// The dequantisation probe reproduces dequant_fp8_block(dtype=float32) bit for bit.
#include "common.cuh"

namespace chronos {

constexpr int kF8Rows = 128, kF8Tok = 32, kF8Step = 64, kF8Threads = 256;
constexpr int kF8Pitch = kF8Step + 8;  // halves per staged token row

__global__ void dequant_fp8_block_kernel(const uint8_t* __restrict__ w, const float* __restrict__ s, float* __restrict__ out, int rows, int cols) {
    const size_t n = (size_t)rows * cols;
    const int sb = (cols + 127) / 128;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / cols, c = i % cols;
        out[i] = __fmul_rn(e4m3_to_f32(w[i]), s[(r / 128) * sb + c / 128]);
    }
}

struct Fp8LinArgs {
    const uint8_t* w;       // [N, K] e4m3
    const float* s;         // [N/128, K/128]
    const void* x;          // [*, K] rows; dtype F32 / BF16 / kDtypeF16Scaled
    int x_dtype;
    const float* xscale;    // [T] power-of-two scale of each row (rows are divided by it on the way to fp16) or NULL
    int row0;               // first row of x / first token
    float* out;             // [T, N] fp32, row t <-> token row0 + t
    int T, N, K;
};

__global__ void __launch_bounds__(kF8Threads) fp8_block_linear_kernel(const Fp8LinArgs a) {
    __shared__ __align__(16) __half xs[2][kF8Tok][kF8Pitch];
    __shared__ float inv_s[kF8Tok];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, q = lane & 3;
    const int n0 = blockIdx.x * kF8Rows, t0 = blockIdx.y * kF8Tok;
    const int nt = min(kF8Tok, a.T - t0);
    if (tid < kF8Tok) inv_s[tid] = (tid < nt && a.xscale != nullptr) ? 1.0f / a.xscale[a.row0 + t0 + tid] : 1.0f;
    __syncthreads();
    // staging: thread -> (token tid / 8, 8 columns (tid % 8) * 8)
    const int st_tok = tid >> 3, st_col = (tid & 7) * 8;
    auto stage = [&](int buf, int k0) {
        uint4 packed = make_uint4(0u, 0u, 0u, 0u);
        if (st_tok < nt) {
            const size_t at = (size_t)(a.row0 + t0 + st_tok) * a.K + k0 + st_col;
            if (a.x_dtype == kDtypeF16Scaled) {
                packed = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(a.x) + at);
            } else {
                float v[8];
                if (a.x_dtype == CHRONOS_DTYPE_BF16) {
                    const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.x) + at);
                    const uint32_t uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) { v[2 * j] = __uint_as_float(uu[j] << 16); v[2 * j + 1] = __uint_as_float(uu[j] & 0xffff0000u); }
                } else {
                    const float4 f0 = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.x) + at);
                    const float4 f1 = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.x) + at + 4);
                    v[0] = f0.x; v[1] = f0.y; v[2] = f0.z; v[3] = f0.w; v[4] = f1.x; v[5] = f1.y; v[6] = f1.z; v[7] = f1.w;
                }
                const float inv = inv_s[st_tok];
                packed.x = pack_f16x2_sat(v[0] * inv, v[1] * inv);
                packed.y = pack_f16x2_sat(v[2] * inv, v[3] * inv);
                packed.z = pack_f16x2_sat(v[4] * inv, v[5] * inv);
                packed.w = pack_f16x2_sat(v[6] * inv, v[7] * inv);
            }
        }
        *reinterpret_cast<uint4*>(&xs[buf][st_tok][st_col]) = packed;
    };
    const uint8_t* w0 = a.w + (size_t)(n0 + warp * 16 + g) * a.K + 16 * q;
    const uint8_t* w1 = w0 + (size_t)8 * a.K;
    const float* srow = a.s + (size_t)blockIdx.x * (a.K / 128);
    float tot[4][4], blk[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int c = 0; c < 4; ++c) { tot[j][c] = 0.0f; blk[j][c] = 0.0f; }
    stage(0, 0);
    uint4 wa = *reinterpret_cast<const uint4*>(w0), wb = *reinterpret_cast<const uint4*>(w1);
    __syncthreads();
    const int n_steps = a.K / kF8Step;
    for (int step = 0; step < n_steps; ++step) {
        const int buf = step & 1;
        uint4 na = wa, nb = wb;
        if (step + 1 < n_steps) {  // next step's operands are requested before this step is multiplied
            stage(buf ^ 1, (step + 1) * kF8Step);
            na = *reinterpret_cast<const uint4*>(w0 + (step + 1) * kF8Step);
            nb = *reinterpret_cast<const uint4*>(w1 + (step + 1) * kF8Step);
        }
        const uint32_t r0[4] = {wa.x, wa.y, wa.z, wa.w}, r1[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
        for (int s4 = 0; s4 < 4; ++s4) {
            // lane (g, q) owns columns 16 q .. 16 q + 15 of the step on both operands; k16 step s4 takes bytes 4 s4 .. 4 s4 + 3
            const uint32_t a0 = e4m3x2_to_f16x2(r0[s4] & 0xffffu), a1 = e4m3x2_to_f16x2(r1[s4] & 0xffffu);
            const uint32_t a2 = e4m3x2_to_f16x2(r0[s4] >> 16), a3 = e4m3x2_to_f16x2(r1[s4] >> 16);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint2 b = *reinterpret_cast<const uint2*>(&xs[buf][8 * j + g][16 * q + 4 * s4]);
                mma_16816(blk[j], a0, a1, a2, a3, b.x, b.y);
            }
        }
        if (step & 1) {  // a 128-column scale block is complete
            const float sc = srow[step >> 1];
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int c = 0; c < 4; ++c) { tot[j][c] = fmaf(sc, blk[j][c], tot[j][c]); blk[j][c] = 0.0f; }
        }
        wa = na;
        wb = nb;
        __syncthreads();
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // tot[j][c]: weight row g (+ 8 for c >= 2), token 8 j + 2 q + (c & 1)
            const int t = 8 * j + 2 * q + (c & 1), n = n0 + warp * 16 + g + (c >> 1) * 8;
            if (t < nt) {
                const float gs = a.xscale != nullptr ? a.xscale[a.row0 + t0 + t] : 1.0f;
                a.out[(size_t)(t0 + t) * a.N + n] = gs * tot[j][c];
            }
        }
}

// act16[t, i] = silu(z[t, i]) * z[t, I + i] as fp16 (saturating)
__global__ void __launch_bounds__(256) shared_swiglu_kernel(const float* __restrict__ z, __half* __restrict__ act, long n, int inter) {
    const long i = ((long)blockIdx.x * 256 + threadIdx.x) * 4;
    if (i >= n) return;
    const long t = i / inter, c = i % inter;
    const float4 zg = *reinterpret_cast<const float4*>(z + t * 2 * inter + c), zu = *reinterpret_cast<const float4*>(z + t * 2 * inter + inter + c);
    const float v[4] = {silu_f32(zg.x) * zu.x, silu_f32(zg.y) * zu.y, silu_f32(zg.z) * zu.z, silu_f32(zg.w) * zu.w};
    store_half4(act + i, v);
}

// y[row0 + t, :] += add[t, :]
__global__ void __launch_bounds__(256) add_rows_kernel(void* __restrict__ y, int y_dtype, const float* __restrict__ add, long n, int hidden, int row0) {
    const long i = ((long)blockIdx.x * 256 + threadIdx.x) * 4;
    if (i >= n) return;
    const float4 v = *reinterpret_cast<const float4*>(add + i);
    const size_t at = (size_t)row0 * hidden + i;
    if (y_dtype == CHRONOS_DTYPE_BF16) {
        __nv_bfloat16* yb = reinterpret_cast<__nv_bfloat16*>(y) + at;
        const uint2 o = *reinterpret_cast<const uint2*>(yb);
        const __nv_bfloat162 a01 = __floats2bfloat162_rn(__uint_as_float(o.x << 16) + v.x, __uint_as_float(o.x & 0xffff0000u) + v.y);
        const __nv_bfloat162 a23 = __floats2bfloat162_rn(__uint_as_float(o.y << 16) + v.z, __uint_as_float(o.y & 0xffff0000u) + v.w);
        uint2 w;
        w.x = *reinterpret_cast<const uint32_t*>(&a01);
        w.y = *reinterpret_cast<const uint32_t*>(&a23);
        *reinterpret_cast<uint2*>(yb) = w;
    } else {
        float4* yf = reinterpret_cast<float4*>(reinterpret_cast<float*>(y) + at);
        float4 o = *yf;
        o.x += v.x; o.y += v.y; o.z += v.z; o.w += v.w;
        *yf = o;
    }
}

int launch_dequant_fp8_block(const uint8_t* w, const float* s, float* out, int rows, int cols, cudaStream_t st) {
    const size_t n = (size_t)rows * cols;
    const int blocks = (int)((n + 255) / 256 < 148 * 16 ? (n + 255) / 256 : 148 * 16);
    dequant_fp8_block_kernel<<<blocks, 256, 0, st>>>(w, s, out, rows, cols);
    return check_launch("dequant_fp8_block");
}

// Shared expert of tokens first .. first + count - 1, added to their rows of y. `tok_scale` [n_tokens] must be ready.
int launch_shared_fp8(const chronos_layer_t& L, const void* x, int x_dtype, const Plan& p, int first, int count, void* y, int y_dtype,
                      cudaStream_t st) {
    if (count <= 0) return CHRONOS_OK;
    const int H = L.hidden, I = L.shared_inter;
    Fp8LinArgs a{};
    a.w = L.sh8_gu_w; a.s = L.sh8_gu_s; a.x = x; a.x_dtype = x_dtype; a.xscale = p.tok_scale; a.row0 = first;
    a.out = p.sh8_z; a.T = count; a.N = 2 * I; a.K = H;
    fp8_block_linear_kernel<<<dim3((unsigned)(a.N / kF8Rows), (unsigned)((count + kF8Tok - 1) / kF8Tok)), kF8Threads, 0, st>>>(a);
    if (int rc = check_launch("shared_fp8 gate_up")) return rc;
    const long n_act = (long)count * I;
    shared_swiglu_kernel<<<(unsigned)((n_act / 4 + 255) / 256), 256, 0, st>>>(p.sh8_z, p.sh8_act, n_act, I);
    if (int rc = check_launch("shared_fp8 swiglu")) return rc;
    Fp8LinArgs d{};
    d.w = L.sh8_dn_w; d.s = L.sh8_dn_s; d.x = p.sh8_act; d.x_dtype = kDtypeF16Scaled; d.xscale = nullptr; d.row0 = 0;
    d.out = p.sh8_y; d.T = count; d.N = H; d.K = I;
    fp8_block_linear_kernel<<<dim3((unsigned)(d.N / kF8Rows), (unsigned)((count + kF8Tok - 1) / kF8Tok)), kF8Threads, 0, st>>>(d);
    if (int rc = check_launch("shared_fp8 down")) return rc;
    const long n_y = (long)count * H;
    add_rows_kernel<<<(unsigned)((n_y / 4 + 255) / 256), 256, 0, st>>>(y, y_dtype, p.sh8_y, n_y, H, first);
    return check_launch("shared_fp8 add");
}

}  // namespace chronos
