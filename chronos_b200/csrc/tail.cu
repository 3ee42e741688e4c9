// Tail lattice: per expert a coarse matrix in natural weight space that the converter adds on top of the unfolded bank
// and the healer (chronos_1t/models/glm53_holo.py:362-366). Codes are 2-bit Lloyd-Max levels with an e4m3 scale per 32
// columns (unpack_2bit_lloyd_max, chronos_1t/models/chronos_moe_block.py:145-157) or 1-bit signs with a scale per 64
// columns (unpack_1bit_rademacher, :212-224): value = level * float(scale).
//
// tail_pass_kernel streams an expert's tail rows once per group of 8 of its pairs and multiplies them by the pairs'
// activations on the tensor cores (mma.sync m16n8k16, fp16): out[pair, row] = g_pair * sum_k T[e, row, k] * x16[pair, k],
// x16 = activations / g_pair in fp16. The consumers (SwiGLU kernel, combine kernel) add the term where they add the healer.
// A warp owns 16 rows; lane (g = lane / 4, q = lane % 4) owns rows g, g + 8 and, per 256-column step, the 64 contiguous
// columns 64 q .. 64 q + 63 (16 bytes of 2-bit codes or 8 bytes of sign bits per row, one vector load): any permutation
// of the contraction index is legal as long as both operands use it, so MMA step s of the 16 takes columns
// 64 q + 4 s .. + 3. Widths that are not a multiple of 256 finish with 64-column steps (16 columns per lane).
#include "common.cuh"

namespace chronos {

__device__ __forceinline__ void mma_16816_t(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                            uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// fp16 bit patterns of the Lloyd-Max levels -1.510417, -0.452780, 0.452780, 1.510417 (round to nearest)
constexpr uint32_t kLloydLo = 0xB73FBE0Bu;  // level 1 in the high half, level 0 in the low half
constexpr uint32_t kLloydHi = 0x3E0B373Fu;  // level 3 high, level 2 low

// two 2-bit codes (bits 0-1 and 2-3 of c4) -> fp16x2 (first code in the low half): one byte permute on the level table
__device__ __forceinline__ uint32_t lloyd2_pair(uint32_t c4) {
    const uint32_t u = (c4 & 3u) | ((c4 & 12u) << 6);  // code 0 at bits 0-1, code 1 at bits 8-9
    return __byte_perm(kLloydLo, kLloydHi, u * 0x22u + 0x1010u);
}
// two sign bits (bit 0, bit 1 of b2; set = +1) -> fp16x2 of +-1
__device__ __forceinline__ uint32_t sign_pair(uint32_t b2) {
    return 0xBC00BC00u ^ (((b2 & 1u) << 15) | ((b2 & 2u) << 30));
}
__device__ __forceinline__ uint32_t e4m3_to_f16x2_dup(uint32_t byte) {
    uint32_t r;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"((uint16_t)(byte | (byte << 8))));
    return r;
}

struct TailArgs {
    const uint8_t* codes; const uint8_t* scales;  // [E, R, K * bits / 8], [E, R, K / block]
    const void* x; int x_dtype;                   // fp16 rows already divided by the pair's scale, or fp32 rows (divided here)
    const int32_t* row_of_pair;                   // token of the pair (gate_up) or NULL: row = pair (down)
    const float* pscale;                          // [P]
    float* out;                                   // [P, R]
    const int32_t* gitem_start; const int32_t* gitem_cnt; const int32_t* pair_expert; const int32_t* counters;
    int R, K, n_experts;
};

// Shared-memory image of the 8 activation rows: every 64-column segment (128 bytes) is followed by 8 bytes of padding
// and rows are 32 bytes (mod 128) apart, so the fragment loads of a warp (8 rows x 4 segments, 8 bytes each) spread over
// the banks as evenly as 256 bytes can.
__host__ __device__ inline int tail_xrow_bytes(int K) {
    const int len = (K / 64) * 136;
    return len + ((32 - len % 128) + 128) % 128;
}
__device__ __forceinline__ int tail_xoff(int k) { return (k >> 6) * 136 + (k & 63) * 2; }

// Code -> fp16 table in shared memory: entry = the 4 values of one code byte (2-bit: 256 entries) or nibble (1-bit: 16
// entries) as two fp16 pairs, 16 copies side by side (entry stride 128 bytes, copy = lane % 16) so that the 32 lookups
// of a warp touch every bank exactly twice - the floor for 256 bytes. One lookup replaces ~12 integer instructions.
template <int BITS>
__device__ __forceinline__ void tail_table_fill(uint8_t* tab, int tid, int nthreads) {
    constexpr int N = BITS == 2 ? 256 : 16;
    for (int i = tid; i < N * 16; i += nthreads) {
        const uint32_t code = (uint32_t)(i >> 4);
        uint2 v;
        if (BITS == 2) { v.x = lloyd2_pair(code); v.y = lloyd2_pair(code >> 4); }
        else { v.x = sign_pair(code); v.y = sign_pair(code >> 2); }
        *reinterpret_cast<uint2*>(tab + (size_t)code * 128 + (i & 15) * 8) = v;
    }
}

template <int BITS>
__device__ __forceinline__ void tail_step4(float (&d)[4], uint32_t w_lo, uint32_t w_hi, uint32_t f_lo, uint32_t f_hi,
                                           const uint8_t* xrow, const uint8_t* tab_lane, int k) {
    // w_*: the codes of 4 columns of rows g / g + 8 in the low bits; k: first of the 4 columns
    constexpr uint32_t M = BITS == 2 ? 0xffu : 0xfu;
    const uint2 lo = *reinterpret_cast<const uint2*>(tab_lane + (size_t)(w_lo & M) * 128);
    const uint2 hi = *reinterpret_cast<const uint2*>(tab_lane + (size_t)(w_hi & M) * 128);
    const uint32_t a0 = hmul2_u32(lo.x, f_lo), a2 = hmul2_u32(lo.y, f_lo);
    const uint32_t a1 = hmul2_u32(hi.x, f_hi), a3 = hmul2_u32(hi.y, f_hi);
    const uint2 b = *reinterpret_cast<const uint2*>(xrow + tail_xoff(k));
    mma_16816_t(d, a0, a1, a2, a3, b.x, b.y);
}

template <int BITS>
__global__ void __launch_bounds__(256) tail_pass_kernel(const TailArgs a) {
    extern __shared__ __align__(128) uint8_t tsm_all[];  // [code table][8 activation rows of K fp16, padded (tail_xrow_bytes)]
    constexpr int TAB = (BITS == 2 ? 256 : 16) * 128;
    uint8_t* tsm = tsm_all + TAB;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, q = lane & 3;
    const int R = a.R, K = a.K, RB = R / 128;
    const int xstride = tail_xrow_bytes(K);
    tail_table_fill<BITS>(tsm_all, tid, 256);  // visible after the first staging barrier below
    const uint8_t* tab_lane = tsm_all + (lane & 15) * 8;
    constexpr int BLK = BITS == 2 ? 32 : 64;
    constexpr int CB = BITS == 2 ? 16 : 8;  // code bytes per lane per 256-column step
    const int K256 = K & ~255;
    const long n_tiles = (long)a.counters[3] * RB;
    const long tile_lo = n_tiles * blockIdx.x / gridDim.x, tile_hi = n_tiles * (blockIdx.x + 1) / gridDim.x;
    int cur_item = -1, cur_chunk = -1;
    for (long tile = tile_lo; tile < tile_hi; ++tile) {
        const int item = (int)(tile / RB), rb = (int)(tile % RB);
        const int start = a.gitem_start[item], cnt = a.gitem_cnt[item];
        const int e = a.pair_expert[start];
        if (e >= a.n_experts) continue;  // shared expert: no tail
        const int row_lo = rb * 128 + warp * 16 + g, row_hi = row_lo + 8;
        const uint8_t* c_lo = a.codes + ((size_t)e * R + row_lo) * (K * BITS / 8);
        const uint8_t* c_hi = a.codes + ((size_t)e * R + row_hi) * (K * BITS / 8);
        const uint8_t* s_lo = a.scales + ((size_t)e * R + row_lo) * (K / BLK);
        const uint8_t* s_hi = a.scales + ((size_t)e * R + row_hi) * (K / BLK);
        for (int chunk = 0; chunk * 8 < cnt; ++chunk) {
            const int c0 = chunk * 8, cn = min(8, cnt - c0);
            if (item != cur_item || chunk != cur_chunk) {  // stage the group's activation rows (block-uniform branch)
                __syncthreads();
                for (int i = tid * 8; i < 8 * K; i += 256 * 8) {
                    const int n = i / K, k = i % K;
                    uint4 v = make_uint4(0u, 0u, 0u, 0u);
                    if (n < cn) {
                        const int pair = start + c0 + n;
                        const size_t row = a.row_of_pair ? (size_t)a.row_of_pair[pair] : (size_t)pair;
                        if (a.x_dtype == kDtypeF16Scaled) {
                            v = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(a.x) + row * K + k);
                        } else {
                            const float gi = 1.0f / a.pscale[pair];
                            const float4* src = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.x) + row * K + k);
                            const float4 f0 = src[0], f1 = src[1];
                            const __half2 h0 = __halves2half2(f32_to_f16_sat(f0.x * gi), f32_to_f16_sat(f0.y * gi));
                            const __half2 h1 = __halves2half2(f32_to_f16_sat(f0.z * gi), f32_to_f16_sat(f0.w * gi));
                            const __half2 h2 = __halves2half2(f32_to_f16_sat(f1.x * gi), f32_to_f16_sat(f1.y * gi));
                            const __half2 h3 = __halves2half2(f32_to_f16_sat(f1.z * gi), f32_to_f16_sat(f1.w * gi));
                            v.x = *reinterpret_cast<const uint32_t*>(&h0); v.y = *reinterpret_cast<const uint32_t*>(&h1);
                            v.z = *reinterpret_cast<const uint32_t*>(&h2); v.w = *reinterpret_cast<const uint32_t*>(&h3);
                        }
                    }
                    uint2* dst = reinterpret_cast<uint2*>(tsm + (size_t)n * xstride + tail_xoff(k));  // 8 columns stay inside a segment
                    dst[0] = make_uint2(v.x, v.y);
                    dst[1] = make_uint2(v.z, v.w);
                }
                __syncthreads();
                cur_item = item;
                cur_chunk = chunk;
            }
            float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            const uint8_t* xrow = tsm + (size_t)g * xstride;
            // 256-column steps: one 16-byte (8-byte) vector of codes and the 2 (1) scale bytes per row and lane
#pragma unroll 2
            for (int k0 = 0; k0 < K256; k0 += 256) {
                uint32_t wl[4], wh[4];
                if (BITS == 2) {
                    const uint4 u = *reinterpret_cast<const uint4*>(c_lo + k0 / 4 + CB * q), v = *reinterpret_cast<const uint4*>(c_hi + k0 / 4 + CB * q);
                    wl[0] = u.x; wl[1] = u.y; wl[2] = u.z; wl[3] = u.w;
                    wh[0] = v.x; wh[1] = v.y; wh[2] = v.z; wh[3] = v.w;
                } else {
                    const uint2 u = *reinterpret_cast<const uint2*>(c_lo + k0 / 8 + CB * q), v = *reinterpret_cast<const uint2*>(c_hi + k0 / 8 + CB * q);
                    wl[0] = u.x & 0xffffu; wl[1] = u.x >> 16; wl[2] = u.y & 0xffffu; wl[3] = u.y >> 16;
                    wh[0] = v.x & 0xffffu; wh[1] = v.x >> 16; wh[2] = v.y & 0xffffu; wh[3] = v.y >> 16;
                }
                uint32_t fl[2], fh[2];
                if (BITS == 2) {  // two blocks of 32 inside the lane's 64 columns
                    const uint32_t sl = *reinterpret_cast<const uint16_t*>(s_lo + k0 / 32 + 2 * q), sh = *reinterpret_cast<const uint16_t*>(s_hi + k0 / 32 + 2 * q);
                    fl[0] = e4m3_to_f16x2_dup(sl & 0xffu); fl[1] = e4m3_to_f16x2_dup(sl >> 8);
                    fh[0] = e4m3_to_f16x2_dup(sh & 0xffu); fh[1] = e4m3_to_f16x2_dup(sh >> 8);
                } else {
                    fl[0] = fl[1] = e4m3_to_f16x2_dup(s_lo[k0 / 64 + q]);
                    fh[0] = fh[1] = e4m3_to_f16x2_dup(s_hi[k0 / 64 + q]);
                }
#pragma unroll
                for (int s = 0; s < 16; ++s) {  // word s / 4 holds the codes of columns 16 (s / 4) .. + 15 of the lane's run
                    const int sh = (s & 3) * (BITS == 2 ? 8 : 4);
                    tail_step4<BITS>(d, wl[s >> 2] >> sh, wh[s >> 2] >> sh, fl[s >> 3], fh[s >> 3], xrow, tab_lane, k0 + 64 * q + 4 * s);
                }
            }
            for (int k0 = K256; k0 < K; k0 += 64) {  // remainder: 16 columns per lane
                uint32_t w_lo, w_hi, f_lo, f_hi;
                if (BITS == 2) {
                    w_lo = *reinterpret_cast<const uint32_t*>(c_lo + k0 / 4 + 4 * q);
                    w_hi = *reinterpret_cast<const uint32_t*>(c_hi + k0 / 4 + 4 * q);
                    f_lo = e4m3_to_f16x2_dup(s_lo[k0 / 32 + (q >> 1)]);
                    f_hi = e4m3_to_f16x2_dup(s_hi[k0 / 32 + (q >> 1)]);
                } else {
                    w_lo = *reinterpret_cast<const uint16_t*>(c_lo + k0 / 8 + 2 * q);
                    w_hi = *reinterpret_cast<const uint16_t*>(c_hi + k0 / 8 + 2 * q);
                    f_lo = e4m3_to_f16x2_dup(s_lo[k0 / 64]);
                    f_hi = e4m3_to_f16x2_dup(s_hi[k0 / 64]);
                }
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    const int sh = s * (BITS == 2 ? 8 : 4);
                    tail_step4<BITS>(d, w_lo >> sh, w_hi >> sh, f_lo, f_hi, xrow, tab_lane, k0 + 16 * q + 4 * s);
                }
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int n = 2 * q + (j & 1), row = j < 2 ? row_lo : row_hi;
                if (n < cn) a.out[(size_t)(start + c0 + n) * R + row] = d[j] * a.pscale[start + c0 + n];
            }
        }
    }
}

int launch_tail_pass(const chronos_layer_t& L, int stage, const void* x, int x_dtype, const Plan& p, cudaStream_t st) {
    const int bits = stage == 0 ? (L.tail_bits & 0xff) : ((L.tail_bits >> 8) & 0xff);
    TailArgs a{};
    a.codes = stage == 0 ? L.tail_gu_p : L.tail_dn_p;
    a.scales = stage == 0 ? L.tail_gu_s : L.tail_dn_s;
    a.x = x;
    a.x_dtype = x_dtype;
    a.row_of_pair = stage == 0 ? p.pair_token : nullptr;
    a.pscale = stage == 0 ? p.pscale_gu : p.pscale_dn;
    a.out = stage == 0 ? p.tail_gu : p.tail_dn;
    a.gitem_start = p.gitem_start;
    a.gitem_cnt = p.gitem_cnt;
    a.pair_expert = p.pair_expert;
    a.counters = p.counters;
    a.R = stage == 0 ? 2 * L.inter : L.hidden;
    a.K = stage == 0 ? L.hidden : L.inter;
    a.n_experts = L.n_experts;
    const size_t smem = (size_t)8 * tail_xrow_bytes(a.K) + (bits == 2 ? 256 : 16) * 128;
    if (smem > 200 * 1024) {
        set_error("tail_pass: %d columns need %zu bytes of shared memory", a.K, smem);
        return CHRONOS_E_SHAPE;
    }
    const int sms = device_sm_count();
    const long max_tiles = (long)p.max_gitems * (a.R / 128);
    const long resident = (long)sms * (smem * 3 <= 222 * 1024 ? 3 : (smem * 2 <= 222 * 1024 ? 2 : 1));
    const unsigned grid = (unsigned)(max_tiles < resident ? max_tiles : resident);
    if (int rc = ensure_dynamic_smem(bits == 2 ? reinterpret_cast<const void*>(tail_pass_kernel<2>) : reinterpret_cast<const void*>(tail_pass_kernel<1>),
                                     smem, "tail_pass")) return rc;
    if (bits == 2) tail_pass_kernel<2><<<grid, 256, smem, st>>>(a);
    else tail_pass_kernel<1><<<grid, 256, smem, st>>>(a);
    return check_launch("tail_pass");
}

// Weight-space probe: out[r, c] += level(code[e, r, c]) * float(scale[e, r, c / block])  (fp32, as the reference adds it)
__global__ void __launch_bounds__(256) tail_add_kernel(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ scales,
                                                       int bits, int rows, int cols, float* __restrict__ out) {
    const long i = (long)blockIdx.x * 256 + threadIdx.x;
    if (i >= (long)rows * cols) return;
    const int r = (int)(i / cols), c = (int)(i % cols);
    float level, scale;
    if (bits == 2) {
        const uint32_t code = (codes[(size_t)r * (cols / 4) + c / 4] >> (2 * (c & 3))) & 3u;
        level = code == 0 ? -1.510417f : (code == 1 ? -0.452780f : (code == 2 ? 0.452780f : 1.510417f));
        scale = e4m3_to_f32(scales[(size_t)r * (cols / 32) + c / 32]);
    } else {
        level = ((codes[(size_t)r * (cols / 8) + c / 8] >> (c & 7)) & 1u) ? 1.0f : -1.0f;
        scale = e4m3_to_f32(scales[(size_t)r * (cols / 64) + c / 64]);
    }
    out[i] += level * scale;
}

int launch_tail_add(const chronos_layer_t& L, int expert, int which, float* out, cudaStream_t st) {
    const int bits = which == 0 ? (L.tail_bits & 0xff) : ((L.tail_bits >> 8) & 0xff);
    const int rows = which == 0 ? 2 * L.inter : L.hidden, cols = which == 0 ? L.hidden : L.inter;
    const int blk = bits == 2 ? 32 : 64;
    const uint8_t* codes = (which == 0 ? L.tail_gu_p : L.tail_dn_p) + (size_t)expert * rows * (cols * bits / 8);
    const uint8_t* scales = (which == 0 ? L.tail_gu_s : L.tail_dn_s) + (size_t)expert * rows * (cols / blk);
    const long n = (long)rows * cols;
    tail_add_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(codes, scales, bits, rows, cols, out);
    return check_launch("tail_add");
}

}  // namespace chronos
