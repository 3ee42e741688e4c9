// Expert-parallel dispatch / combine helpers: the device side of the deduplicated all-to-all.
//
// A token's hidden row travels ONCE to every rank that owns at least one of its top-k experts (not once per expert),
// together with its expert ids local to that rank and their gates; after the expert pass each rank returns ONE partial
// sum row per received token, and the home rank adds the partial rows in rank order. The exchange itself is a
// collective with equal, fixed-capacity blocks per peer (no sizes ever cross the host, the step stays stream-ordered);
// these kernels fill and read the blocks:
//   ep_plan_kernel       per destination rank: which local tokens go there and at which position of the block
//                        (position = number of earlier tokens that go there too: deterministic), the block's row count
//   ep_pack_rows_kernel  copies the rows and writes the per-row metadata
//   ep_unpack_meta_kernel received metadata -> routing lists (ids local to this rank, gates) of the received rows
//   ep_combine_kernel    y[t] = extra[t] + sum over ranks d (in order) of the partial row d returned for token t
// The reference has no distributed path (single device); the partitioning is by slot, never inside a slot.
#include <algorithm>

#include "common.cuh"

namespace chronos {

constexpr int kEpPlanThreads = 1024;

// meta: int32 [world, capacity + 1, 2 * top_k + 2]; row p < capacity: [0] source token, [1 .. k] expert ids local to
// the destination (-1: not owned there), [k + 1 .. 2k] gate bits; row `capacity`: [0] = rows used in the block.
__global__ void __launch_bounds__(kEpPlanThreads) ep_plan_kernel(const int32_t* __restrict__ ids, int n_tokens, int top_k,
                                                                 int experts_per_rank, int capacity, int32_t* __restrict__ meta,
                                                                 long meta_block_ints, int32_t* __restrict__ slot_of, int world,
                                                                 int32_t* __restrict__ overflow) {
    __shared__ int warp_tot[kEpPlanThreads / 32 + 1];
    const int d = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int lo = d * experts_per_rank, hi = lo + experts_per_rank;
    int carry = 0;
    for (int base = 0; base < n_tokens; base += kEpPlanThreads) {
        const int t = base + tid;
        int flag = 0;
        if (t < n_tokens)
            for (int j = 0; j < top_k; ++j) {
                const int e = ids[(size_t)t * top_k + j];
                flag |= (e >= lo && e < hi);
            }
        int inc = flag;
#pragma unroll
        for (int s = 1; s < 32; s <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, inc, s);
            if (lane >= s) inc += o;
        }
        __syncthreads();  // warp_tot of the previous chunk has been read
        if (lane == 31) warp_tot[warp] = inc;
        __syncthreads();
        if (warp == 0) {
            const int w = warp_tot[lane];
            int winc = w;
#pragma unroll
            for (int s = 1; s < 32; s <<= 1) {
                const int o = __shfl_up_sync(0xffffffffu, winc, s);
                if (lane >= s) winc += o;
            }
            warp_tot[lane] = winc - w;
            if (lane == 31) warp_tot[32] = winc;
        }
        __syncthreads();
        const int pos = carry + warp_tot[warp] + inc - flag;
        if (t < n_tokens) slot_of[(size_t)t * world + d] = (flag && pos < capacity) ? pos : -1;
        if (flag && pos >= capacity) atomicOr(overflow, 1);  // the block is full: the caller learns of it and repeats the step
        carry += warp_tot[32];
    }
    if (tid == 0) meta[(size_t)d * meta_block_ints + (size_t)capacity * (2 * top_k + 2)] = min(carry, capacity);
}

__global__ void __launch_bounds__(128) ep_pack_rows_kernel(const uint4* __restrict__ x, int row_vec16, const int32_t* __restrict__ ids,
                                                           const float* __restrict__ gates, int top_k, int experts_per_rank, int capacity,
                                                           const int32_t* __restrict__ slot_of, int world, uint4* __restrict__ send_rows,
                                                           int block_rows, int32_t* __restrict__ meta, long meta_block_ints) {
    const int t = blockIdx.x, d = blockIdx.y;
    const int p = slot_of[(size_t)t * world + d];
    if (p < 0) return;
    const uint4* src = x + (size_t)t * row_vec16;
    uint4* dst = send_rows + ((size_t)d * block_rows + p) * row_vec16;
    for (int i = threadIdx.x; i < row_vec16; i += 128) dst[i] = src[i];
    const int m = 2 * top_k + 2;
    int32_t* mrow = meta + (size_t)d * meta_block_ints + (size_t)p * m;
    if (threadIdx.x == 0) mrow[0] = t;
    if (threadIdx.x < top_k) {
        const int e = ids[(size_t)t * top_k + threadIdx.x] - d * experts_per_rank;
        const bool mine = e >= 0 && e < experts_per_rank;
        mrow[1 + threadIdx.x] = mine ? e : -1;
        mrow[1 + top_k + threadIdx.x] = mine ? __float_as_int(gates[(size_t)t * top_k + threadIdx.x]) : 0;
    }
}

// Rows of the routing lists: world blocks of block_rows rows (rows at and past `capacity` of a block, where a merged
// exchange buffer carries the metadata itself, get no expert), then tail_rows rows without experts (the home tokens).
__global__ void __launch_bounds__(256) ep_unpack_meta_kernel(const int32_t* __restrict__ meta, long meta_block_ints, int world, int capacity,
                                                             int block_rows, int tail_rows, int top_k, int32_t* __restrict__ ids_out,
                                                             float* __restrict__ gates_out) {
    const long i = (long)blockIdx.x * 256 + threadIdx.x;  // over (world * block_rows + tail_rows) * top_k
    if (i >= ((long)world * block_rows + tail_rows) * top_k) return;
    const int j = (int)(i % top_k);
    const long row = i / top_k;
    const int s = (int)(row / block_rows), p = (int)(row % block_rows);
    const int m = 2 * top_k + 2;
    bool valid = false;
    const int32_t* blk = meta;
    if (s < world && p < capacity) {
        blk = meta + (size_t)s * meta_block_ints;
        valid = p < blk[(size_t)capacity * m];
    }
    ids_out[i] = valid ? blk[(size_t)p * m + 1 + j] : -1;
    gates_out[i] = valid ? __int_as_float(blk[(size_t)p * m + 1 + top_k + j]) : 0.0f;
}

template <typename T>
__device__ __forceinline__ float4 ld4(const T* p);
template <>
__device__ __forceinline__ float4 ld4<float>(const float* p) { return *reinterpret_cast<const float4*>(p); }
template <>
__device__ __forceinline__ float4 ld4<__nv_bfloat16>(const __nv_bfloat16* p) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    return make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u), __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xffff0000u));
}

template <typename TIN>
__global__ void __launch_bounds__(256) ep_combine_kernel(const TIN* __restrict__ back, const int32_t* __restrict__ slot_of,
                                                         const TIN* __restrict__ extra, int hidden, int world, int block_rows,
                                                         void* __restrict__ y, int y_dtype) {
    const int t = blockIdx.x, i0 = (blockIdx.y * 256 + threadIdx.x) * 4;
    if (i0 >= hidden) return;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (extra != nullptr) acc = ld4<TIN>(extra + (size_t)t * hidden + i0);
    for (int d = 0; d < world; ++d) {  // rank order: the same sum whatever the arrival order was
        const int p = slot_of[(size_t)t * world + d];
        if (p < 0) continue;
        const float4 v = ld4<TIN>(back + ((size_t)d * block_rows + p) * hidden + i0);
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    if (y_dtype == CHRONOS_DTYPE_BF16) {
        const __nv_bfloat162 a01 = __floats2bfloat162_rn(acc.x, acc.y), a23 = __floats2bfloat162_rn(acc.z, acc.w);
        uint2 o;
        o.x = *reinterpret_cast<const uint32_t*>(&a01);
        o.y = *reinterpret_cast<const uint32_t*>(&a23);
        *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(y) + (size_t)t * hidden + i0) = o;
    } else {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(y) + (size_t)t * hidden + i0) = acc;
    }
}

// ---------------------------------------------------------------------------------------------------------------
// The same exchange without a collective: every rank holds a receive buffer that its peers can write (symmetric memory
// over NVLink), laid out as world blocks of block_rows rows (block s = what rank s sent: its rows, then the metadata).
// The pack kernels store straight into the peers' buffers (block index = this rank), a barrier kernel then tells every
// peer "my stores of this epoch are done" and waits for the same word from each of them.
//   peer_bases[d]  base of rank d's receive buffer as mapped into this process (d = this rank: the local buffer)
//   pads[d]        a few 32-bit words in rank d's memory that peers may write: word s = last epoch rank s finished
// Plain peer stores and loads only. The wait is bounded; on expiry the status word gets kStatusEpBarrierTimeout.
// ---------------------------------------------------------------------------------------------------------------
constexpr uint32_t kEpBarrierPolls = 1u << 22;  // ~0.25 us each: about a second

__global__ void __launch_bounds__(kEpPlanThreads) ep_plan_peer_kernel(const int32_t* __restrict__ ids, int n_tokens, int top_k,
                                                                      int experts_per_rank, int capacity, uint8_t* const* __restrict__ peer_bases,
                                                                      int my_rank, size_t block_bytes, size_t meta_off, int32_t* __restrict__ slot_of,
                                                                      int world, int32_t* __restrict__ overflow) {
    __shared__ int warp_tot[kEpPlanThreads / 32 + 1];
    const int d = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int lo = d * experts_per_rank, hi = lo + experts_per_rank;
    int carry = 0;
    for (int base = 0; base < n_tokens; base += kEpPlanThreads) {
        const int t = base + tid;
        int flag = 0;
        if (t < n_tokens)
            for (int j = 0; j < top_k; ++j) {
                const int e = ids[(size_t)t * top_k + j];
                flag |= (e >= lo && e < hi);
            }
        int inc = flag;
#pragma unroll
        for (int s = 1; s < 32; s <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, inc, s);
            if (lane >= s) inc += o;
        }
        __syncthreads();  // warp_tot of the previous chunk has been read
        if (lane == 31) warp_tot[warp] = inc;
        __syncthreads();
        if (warp == 0) {
            const int w = warp_tot[lane];
            int winc = w;
#pragma unroll
            for (int s = 1; s < 32; s <<= 1) {
                const int o = __shfl_up_sync(0xffffffffu, winc, s);
                if (lane >= s) winc += o;
            }
            warp_tot[lane] = winc - w;
            if (lane == 31) warp_tot[32] = winc;
        }
        __syncthreads();
        const int pos = carry + warp_tot[warp] + inc - flag;
        if (t < n_tokens) slot_of[(size_t)t * world + d] = (flag && pos < capacity) ? pos : -1;
        if (flag && pos >= capacity) atomicOr(overflow, 1);
        carry += warp_tot[32];
    }
    if (tid == 0) {
        int32_t* meta = reinterpret_cast<int32_t*>(peer_bases[d] + (size_t)my_rank * block_bytes + meta_off);
        meta[(size_t)capacity * (2 * top_k + 2)] = min(carry, capacity);
    }
}

__global__ void __launch_bounds__(128) ep_pack_rows_peer_kernel(const uint4* __restrict__ x, int row_vec16, const int32_t* __restrict__ ids,
                                                                const float* __restrict__ gates, int top_k, int experts_per_rank,
                                                                const int32_t* __restrict__ slot_of, int world,
                                                                uint8_t* const* __restrict__ peer_bases, int my_rank, size_t block_bytes,
                                                                size_t meta_off) {
    const int t = blockIdx.x, d = blockIdx.y;
    const uint4* src = x + (size_t)t * row_vec16;
    if (d == world) {  // the token's own copy behind the blocks of the local buffer (it takes the shared expert at home)
        uint4* home = reinterpret_cast<uint4*>(peer_bases[my_rank] + (size_t)world * block_bytes) + (size_t)t * row_vec16;
        for (int i = threadIdx.x; i < row_vec16; i += 128) home[i] = src[i];
        return;
    }
    const int p = slot_of[(size_t)t * world + d];
    if (p < 0) return;
    uint8_t* block = peer_bases[d] + (size_t)my_rank * block_bytes;
    uint4* dst = reinterpret_cast<uint4*>(block) + (size_t)p * row_vec16;
    for (int i = threadIdx.x; i < row_vec16; i += 128) dst[i] = src[i];
    const int m = 2 * top_k + 2;
    int32_t* mrow = reinterpret_cast<int32_t*>(block + meta_off) + (size_t)p * m;
    if (threadIdx.x == 0) mrow[0] = t;
    if (threadIdx.x < top_k) {
        const int e = ids[(size_t)t * top_k + threadIdx.x] - d * experts_per_rank;
        const bool mine = e >= 0 && e < experts_per_rank;
        mrow[1 + threadIdx.x] = mine ? e : -1;
        mrow[1 + top_k + threadIdx.x] = mine ? __float_as_int(gates[(size_t)t * top_k + threadIdx.x]) : 0;
    }
}

// The way back: block s of the local partial-sum rows (rows of the tokens rank s sent; their number is the count word of
// the metadata rank s sent along) goes into block `my_rank` of rank s's return buffer.
__global__ void __launch_bounds__(256) ep_send_back_peer_kernel(const uint4* __restrict__ part, int row_vec16, int block_rows,
                                                                const uint8_t* __restrict__ recv_base, size_t block_bytes, size_t meta_off,
                                                                int capacity, int top_k, uint8_t* const* __restrict__ peer_back, int my_rank) {
    const int s = blockIdx.y;
    const int cnt = reinterpret_cast<const int32_t*>(recv_base + (size_t)s * block_bytes + meta_off)[(size_t)capacity * (2 * top_k + 2)];
    const uint4* src = part + (size_t)s * block_rows * row_vec16;
    uint4* dst = reinterpret_cast<uint4*>(peer_back[s] + (size_t)my_rank * block_bytes);
    const long n = (long)min(cnt, capacity) * row_vec16;
    for (long i = (long)blockIdx.x * 256 + threadIdx.x; i < n; i += (long)gridDim.x * 256) dst[i] = src[i];
}

__global__ void __launch_bounds__(1024) ep_barrier_kernel(uint32_t* const* __restrict__ pads, int my_rank, int world, uint32_t epoch,
                                                          int32_t* __restrict__ status) {
    const int d = threadIdx.x;
    if (d >= world) return;
    __threadfence_system();  // the stores of the kernels before this one are visible to the peers before the word below
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(pads[d] + my_rank), "r"(epoch) : "memory");
    const uint32_t* mine = pads[my_rank] + d;
    bool ok = false;
    for (uint32_t poll = 0; poll < kEpBarrierPolls; ++poll) {
        uint32_t seen;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(seen) : "l"(mine) : "memory");
        if ((int32_t)(seen - epoch) >= 0) { ok = true; break; }
        __nanosleep(200);
    }
    if (!ok) atomicOr(status, kStatusEpBarrierTimeout);
}

int launch_ep_pack_peer(const void* x, int x_dtype, const int32_t* ids, const float* gates, int n_tokens, int top_k, int hidden,
                        int world, int experts_per_rank, int capacity, void* const* peer_bases, int my_rank, int block_rows,
                        int32_t* slot_of, int32_t* overflow, cudaStream_t st) {
    if (n_tokens <= 0) return CHRONOS_OK;
    const size_t row_bytes = (size_t)hidden * (x_dtype == CHRONOS_DTYPE_BF16 ? 2 : 4);
    const size_t block_bytes = (size_t)block_rows * row_bytes, meta_off = (size_t)capacity * row_bytes;
    uint8_t* const* bases = reinterpret_cast<uint8_t* const*>(peer_bases);
    ep_plan_peer_kernel<<<(unsigned)world, kEpPlanThreads, 0, st>>>(ids, n_tokens, top_k, experts_per_rank, capacity, bases, my_rank, block_bytes,
                                                                   meta_off, slot_of, world, overflow);
    if (int rc = check_launch("ep_plan_peer")) return rc;
    ep_pack_rows_peer_kernel<<<dim3((unsigned)n_tokens, (unsigned)world + 1), 128, 0, st>>>(reinterpret_cast<const uint4*>(x), (int)(row_bytes / 16), ids,
                                                                                       gates, top_k, experts_per_rank, slot_of, world, bases, my_rank,
                                                                                       block_bytes, meta_off);
    return check_launch("ep_pack_rows_peer");
}

int launch_ep_send_back_peer(const void* part, int dtype, int hidden, int world, int block_rows, int capacity, int top_k, const void* recv_base,
                             void* const* peer_back, int my_rank, cudaStream_t st) {
    const size_t row_bytes = (size_t)hidden * (dtype == CHRONOS_DTYPE_BF16 ? 2 : 4);
    const size_t block_bytes = (size_t)block_rows * row_bytes, meta_off = (size_t)capacity * row_bytes;
    const int per_peer = std::max(1, 4 * device_sm_count() / world);
    ep_send_back_peer_kernel<<<dim3((unsigned)per_peer, (unsigned)world), 256, 0, st>>>(
        reinterpret_cast<const uint4*>(part), (int)(row_bytes / 16), block_rows, reinterpret_cast<const uint8_t*>(recv_base), block_bytes, meta_off,
        capacity, top_k, reinterpret_cast<uint8_t* const*>(peer_back), my_rank);
    return check_launch("ep_send_back_peer");
}

int launch_ep_barrier(void* const* pads, int my_rank, int world, uint32_t epoch, int32_t* status, cudaStream_t st) {
    ep_barrier_kernel<<<1, 1024, 0, st>>>(reinterpret_cast<uint32_t* const*>(pads), my_rank, world, epoch, status);
    return check_launch("ep_barrier");
}

int launch_ep_pack(const void* x, int x_dtype, const int32_t* ids, const float* gates, int n_tokens, int top_k, int hidden,
                   int world, int experts_per_rank, int capacity, void* send_rows, int32_t* send_meta, int32_t* slot_of,
                   int32_t* overflow, int block_rows, long meta_block_ints, cudaStream_t st) {
    if (n_tokens <= 0) return CHRONOS_OK;
    if (block_rows <= 0) block_rows = capacity;
    if (meta_block_ints <= 0) meta_block_ints = (long)(capacity + 1) * (2 * top_k + 2);
    ep_plan_kernel<<<(unsigned)world, kEpPlanThreads, 0, st>>>(ids, n_tokens, top_k, experts_per_rank, capacity, send_meta, meta_block_ints,
                                                              slot_of, world, overflow);
    if (int rc = check_launch("ep_plan")) return rc;
    const int row_vec16 = hidden * (x_dtype == CHRONOS_DTYPE_BF16 ? 2 : 4) / 16;
    ep_pack_rows_kernel<<<dim3((unsigned)n_tokens, (unsigned)world), 128, 0, st>>>(reinterpret_cast<const uint4*>(x), row_vec16, ids, gates, top_k,
                                                                                  experts_per_rank, capacity, slot_of, world,
                                                                                  reinterpret_cast<uint4*>(send_rows), block_rows, send_meta,
                                                                                  meta_block_ints);
    return check_launch("ep_pack_rows");
}

int launch_ep_unpack_meta(const int32_t* meta, int world, int capacity, int top_k, int32_t* ids_out, float* gates_out, int block_rows,
                          long meta_block_ints, int tail_rows, cudaStream_t st) {
    if (block_rows <= 0) block_rows = capacity;
    if (meta_block_ints <= 0) meta_block_ints = (long)(capacity + 1) * (2 * top_k + 2);
    const long n = ((long)world * block_rows + tail_rows) * top_k;
    if (n <= 0) return CHRONOS_OK;
    ep_unpack_meta_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(meta, meta_block_ints, world, capacity, block_rows, tail_rows, top_k,
                                                                      ids_out, gates_out);
    return check_launch("ep_unpack_meta");
}

int launch_ep_combine(const void* back, int dtype, const int32_t* slot_of, const void* extra, int n_tokens, int hidden, int world,
                      int capacity, void* y, int y_dtype, int block_rows, cudaStream_t st) {
    if (n_tokens <= 0) return CHRONOS_OK;
    if (block_rows <= 0) block_rows = capacity;
    const dim3 grid((unsigned)n_tokens, (unsigned)((hidden / 4 + 255) / 256));
    if (dtype == CHRONOS_DTYPE_BF16)
        ep_combine_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(back), slot_of,
                                                              reinterpret_cast<const __nv_bfloat16*>(extra), hidden, world, block_rows, y, y_dtype);
    else
        ep_combine_kernel<float><<<grid, 256, 0, st>>>(reinterpret_cast<const float*>(back), slot_of, reinterpret_cast<const float*>(extra),
                                                      hidden, world, block_rows, y, y_dtype);
    return check_launch("ep_combine");
}

}  // namespace chronos
