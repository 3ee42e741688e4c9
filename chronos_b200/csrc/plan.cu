// Batch coalescing on the device: sorts (token, expert) routing entries by expert, so that the entries of one slot
// are contiguous, and cuts them into work items: up to 8 pairs that share one pass over the slot's bank (streaming
// regimes) and up to 128 (64 in the FP4 tensor regime) pairs of one expert.
// Takes the role of `torch.unique` + per-expert gathers (chronos_1t/models/glm5_chronos_moe.py:508-522) and of
// the argsort/unique_consecutive grouping (chronos_1t/models/glm53_chronos_moe.py:456-459) with no host round trip.
// For decode-sized batches the top-k selection runs inside the same launch (one warp per token).
#include "common.cuh"

namespace chronos {

constexpr int kPlanThreads = 1024;
constexpr int kPlanWarps = kPlanThreads / 32;
constexpr int kPlanMaxBins = 1024 + 1;  // experts + the shared-expert bin
constexpr int kPlanBatch = 8;            // routing entries a thread reads ahead

// Exclusive scan over the block: every thread passes its value and gets the sum of the values of lower threads;
// `total` receives the block sum. Warp shuffles inside the warps, warp 0 scans the warp totals.
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_tot /*[kPlanWarps + 1]*/, int& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int inc = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, inc, d);
        if (lane >= d) inc += o;
    }
    __syncthreads();  // warp_tot may still be read from a previous call
    if (lane == 31) warp_tot[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        const int w = lane < kPlanWarps ? warp_tot[lane] : 0;  // fewer than 32 warps: the other lanes scan zeros
        int winc = w;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, winc, d);
            if (lane >= d) winc += o;
        }
        if (lane < kPlanWarps) warp_tot[lane] = winc - w;  // exclusive prefix of the warp totals
        if (lane == 31) warp_tot[kPlanWarps] = winc;
    }
    __syncthreads();
    total = warp_tot[kPlanWarps];
    return warp_tot[warp] + inc - v;
}

__global__ void __launch_bounds__(kPlanThreads) plan_kernel(const int32_t* __restrict__ ids_in, int n_tokens, int top_k,
                                                            int n_experts, int group_size, int n_slots, int with_shared,
                                                            int reset_status, int scatter_here, TopkArgs tk, Plan p) {
    __shared__ int cnt[kPlanMaxBins + 1];
    __shared__ int off[kPlanMaxBins + 1];
    __shared__ int cur[kPlanMaxBins + 1];
    __shared__ int warp_tot[kPlanWarps + 1];
    const int tid = threadIdx.x;
    const int n_bins = n_experts + 1;
    const int n_entries = n_tokens * top_k;
    for (int i = tid; i <= n_bins; i += kPlanThreads) { cnt[i] = 0; cur[i] = 0; }
    const int32_t* ids = ids_in;
    if (tk.logits != nullptr) {  // fused top-k: one warp per token (decode-sized batches only)
        for (int t = tid >> 5; t < n_tokens; t += kPlanWarps) topk_one_token(tk, t, tid & 31);
        ids = tk.ids;
    }
    __syncthreads();  // also orders the ids written above (global memory, same block) before they are read back
    // popular experts (skewed routing) would serialise thousands of shared-memory atomics on one counter: the lanes of a
    // warp that hold the same expert elect a leader, which adds their number once
    const int lane = tid & 31;
    // (the entries are read kPlanBatch at a time: one CTA walks the whole list, and a global load per step would make
    // the walk a chain of memory round trips)
    for (int i0 = tid - lane; i0 < n_entries; i0 += kPlanThreads * kPlanBatch) {
        int ev[kPlanBatch];
#pragma unroll
        for (int b = 0; b < kPlanBatch; ++b) {
            const int i = i0 + b * kPlanThreads + lane;
            ev[b] = i < n_entries ? ids[i] : -1;
        }
#pragma unroll
        for (int b = 0; b < kPlanBatch; ++b) {
            if (i0 + b * kPlanThreads >= n_entries) break;  // warp-uniform
            const int e = (ev[b] < 0 || ev[b] >= n_experts) ? -1 : ev[b];
            const unsigned same = __match_any_sync(0xffffffffu, e);
            if (e >= 0 && lane == __ffs(same) - 1) atomicAdd(&cnt[e], __popc(same));
        }
    }
    if (tid == 0 && with_shared) cnt[n_experts] = p.shared_n;  // tokens shared_lo .. shared_lo + shared_n - 1
    __syncthreads();
    // exclusive scan of cnt[0 .. n_bins) (n_bins <= 1025): chunks of 1024 with a carry
    int carry = 0;
    for (int base = 0; base < n_bins; base += kPlanThreads) {
        const int idx = base + tid;
        const int v = idx < n_bins ? cnt[idx] : 0;
        int total;
        const int ex = block_exclusive_scan(v, warp_tot, total);
        if (idx < n_bins) off[idx] = carry + ex;
        carry += total;
    }
    if (tid == 0) off[n_bins] = carry;
    __syncthreads();
    for (int i = tid; i <= n_bins; i += kPlanThreads) { p.offsets[i] = off[i]; p.cursor[i] = 0; }
    // scatter entries to their sorted position (order inside an expert is arbitrary: no result depends on it); a large
    // batch leaves that to plan_scatter_kernel: the scattered stores of one SM are what bounds this loop
    for (int i0 = tid - lane; scatter_here && i0 < n_entries; i0 += kPlanThreads * kPlanBatch) {
        int ev[kPlanBatch];
#pragma unroll
        for (int b = 0; b < kPlanBatch; ++b) {
            const int i = i0 + b * kPlanThreads + lane;
            ev[b] = i < n_entries ? ids[i] : -1;
        }
#pragma unroll
        for (int b = 0; b < kPlanBatch; ++b) {
            if (i0 + b * kPlanThreads >= n_entries) break;  // warp-uniform
            const int i = i0 + b * kPlanThreads + lane;
            const int e = (ev[b] < 0 || ev[b] >= n_experts) ? -1 : ev[b];
            const unsigned same = __match_any_sync(0xffffffffu, e);
            const int leader = __ffs(same) - 1;
            int first = 0;
            if (e >= 0 && lane == leader) first = atomicAdd(&cur[e], __popc(same));
            first = __shfl_sync(0xffffffffu, first, leader);
            int pos = -1;
            if (e >= 0) {
                pos = off[e] + first + __popc(same & ((1u << lane) - 1u));
                p.pair_token[pos] = i / top_k;
                p.pair_expert[pos] = e;
            }
            if (i < n_entries) p.pos_of[i] = pos;
        }
    }
    if (with_shared)
        for (int t = tid; t < p.shared_n; t += kPlanThreads) {
            p.pair_token[off[n_experts] + t] = p.shared_lo + t;
            p.pair_expert[off[n_experts] + t] = n_experts;
        }
    // streaming work items: slot s owns sorted pairs [off[s*K], off[(s+1)*K]); the shared expert is slot n_slots.
    // First the number of items before each slot (into `cur`, free by now), then one thread per ITEM, which finds its slot
    // by bisection: a slot with thousands of pairs does not leave its items to one thread.
    __syncthreads();
    carry = 0;
    const int n_vslots = n_slots + 1;
    auto slot_range = [&](int s, int& lo, int& hi) {
        lo = 0; hi = 0;
        if (s < n_slots) { lo = off[s * group_size]; hi = off[(s + 1) * group_size]; }
        else if (s == n_slots) { lo = off[n_experts]; hi = off[n_bins]; }
    };
    auto owner_of = [&](const int* first, int n, int it) {  // largest s < n with first[s] <= it
        int a = 0, b = n - 1;
        while (a < b) {
            const int m = (a + b + 1) >> 1;
            if (first[m] <= it) a = m; else b = m - 1;
        }
        return a;
    };
    for (int base = 0; base < n_vslots; base += kPlanThreads) {
        const int s = base + tid;
        int lo, hi;
        slot_range(s, lo, hi);
        const int ni = (hi - lo + kPairsPerItem - 1) / kPairsPerItem;
        int total;
        const int first = carry + block_exclusive_scan(ni, warp_tot, total);
        if (s < n_vslots) cur[s] = first;
        carry += total;
    }
    const int n_items_total = carry;
    __syncthreads();
    for (int it = tid; it < min(n_items_total, p.max_items); it += kPlanThreads) {
        const int s = owner_of(cur, n_vslots, it), q = it - cur[s];
        int lo, hi;
        slot_range(s, lo, hi);
        p.item_start[it] = lo + q * kPairsPerItem;
        p.item_cnt[it] = min(kPairsPerItem, hi - lo - q * kPairsPerItem);
        p.item_slot[it] = s;
    }
    // tensor-core work items: expert e (bin n_experts = shared expert) owns sorted pairs [off[e], off[e+1]), cut into
    // blocks of gitem_pairs (128, or 64 in the FP4 tensor regime) so that one MMA tile never mixes experts
    carry = 0;
    const int gp = p.gitem_pairs;
    for (int base = 0; base < n_bins; base += kPlanThreads) {
        const int e = base + tid;
        const int ni = e < n_bins ? (off[e + 1] - off[e] + gp - 1) / gp : 0;
        int total;
        const int first = carry + block_exclusive_scan(ni, warp_tot, total);
        if (e < n_bins) cnt[e] = first;  // the counts are no longer needed: off holds their prefix sums
        carry += total;
    }
    __syncthreads();
    for (int it = tid; it < min(carry, p.max_gitems); it += kPlanThreads) {
        const int e = owner_of(cnt, n_bins, it), q = it - cnt[e];
        const int lo = off[e], hi = off[e + 1];
        p.gitem_start[it] = lo + q * gp;
        p.gitem_cnt[it] = min(gp, hi - lo - q * gp);
        p.gitem_slot[it] = e < n_experts ? e / group_size : n_slots;
    }
    if (tid == 0) {
        p.counters[4] = min(cnt[n_experts], p.max_gitems);  // first tensor-core work item of the shared expert (= the total without one)
        p.counters[3] = min(carry, p.max_gitems);
        p.counters[0] = min(n_items_total, p.max_items);
        p.counters[1] = off[n_bins];
        if (reset_status) p.counters[2] = 0;  // otherwise the caller cleared it before the router ran
    }
}

// Scatter of a large batch: every CTA places a slice of the routing entries at offsets[e] + (a ticket from the expert's
// cursor); lanes of a warp that hold the same expert take their tickets with one atomic.
__global__ void __launch_bounds__(256) plan_scatter_kernel(const int32_t* __restrict__ ids, int n_entries, int top_k, int n_experts, Plan p) {
    const int lane = threadIdx.x & 31;
    for (int i0 = blockIdx.x * 256 + threadIdx.x - lane; i0 < n_entries; i0 += gridDim.x * 256) {
        const int i = i0 + lane;
        int e = i < n_entries ? ids[i] : -1;
        if (e < 0 || e >= n_experts) e = -1;
        const unsigned same = __match_any_sync(0xffffffffu, e);
        const int leader = __ffs(same) - 1;
        int first = 0;
        if (e >= 0 && lane == leader) first = atomicAdd(&p.cursor[e], __popc(same));
        first = __shfl_sync(0xffffffffu, first, leader);
        int pos = -1;
        if (e >= 0) {
            pos = p.offsets[e] + first + __popc(same & ((1u << lane) - 1u));
            p.pair_token[pos] = i / top_k;
            p.pair_expert[pos] = e;
        }
        if (i < n_entries) p.pos_of[i] = pos;
    }
}

int launch_plan(const chronos_layer_t& L, const int32_t* ids, int n_tokens, int with_shared, int reset_status,
                const TopkArgs& tk, const Plan& p, cudaStream_t st) {
    const int n_entries = n_tokens * L.top_k;
    const bool split = tk.logits == nullptr && n_entries >= 8192;
    plan_kernel<<<1, kPlanThreads, 0, st>>>(ids, n_tokens, L.top_k, L.n_experts, L.group_size, L.n_slots,
                                           with_shared && L.shared_inter > 0, reset_status, split ? 0 : 1, tk, p);
    if (int rc = check_launch("plan")) return rc;
    if (!split) return CHRONOS_OK;
    const int most = (n_entries + 255) / 256, resident = 4 * device_sm_count();
    plan_scatter_kernel<<<(unsigned)(most < resident ? most : resident), 256, 0, st>>>(ids, n_entries, L.top_k, L.n_experts, p);
    return check_launch("plan_scatter");
}

}  // namespace chronos
