// Batch coalescing on the device: sorts (token, expert) routing entries by expert, so that the entries of one slot
// are contiguous, and cuts them into work items of up to 8 pairs that share one pass over the slot's bank.
// Takes the role of `torch.unique` + per-expert gathers (chronos_1t/models/glm5_chronos_moe.py:508-522) and of
// the argsort/unique_consecutive grouping (chronos_1t/models/glm53_chronos_moe.py:456-459) with no host round trip.
#include "common.cuh"

namespace chronos {

constexpr int kPlanThreads = 1024;
constexpr int kPlanMaxBins = 1024 + 1;  // experts + the shared-expert bin

__global__ void __launch_bounds__(kPlanThreads) plan_kernel(const int32_t* __restrict__ ids, int n_tokens, int top_k,
                                                            int n_experts, int group_size, int n_slots, int with_shared,
                                                            const void* __restrict__ x, int x_dtype, int hidden,
                                                            int reset_status, Plan p) {
    __shared__ int cnt[kPlanMaxBins + 1];
    __shared__ int off[kPlanMaxBins + 1];
    __shared__ int cur[kPlanMaxBins + 1];
    __shared__ int scan[2][kPlanThreads + 1];
    const int tid = threadIdx.x;
    const int n_bins = n_experts + 1;
    const int n_entries = n_tokens * top_k;
    for (int i = tid; i <= n_bins; i += kPlanThreads) { cnt[i] = 0; cur[i] = 0; }
    __syncthreads();
    for (int i = tid; i < n_entries; i += kPlanThreads) {
        const int e = ids[i];
        if (e >= 0 && e < n_experts) atomicAdd(&cnt[e], 1);
    }
    if (tid == 0 && with_shared) cnt[n_experts] = n_tokens;
    __syncthreads();
    // exclusive scan of cnt[0 .. n_bins) (n_bins <= 1025): chunked Hillis-Steele over 1024 + carry
    int carry = 0;
    for (int base = 0; base < n_bins; base += kPlanThreads) {
        const int idx = base + tid;
        const int v = idx < n_bins ? cnt[idx] : 0;
        int src = 0;
        scan[0][tid] = v;
        __syncthreads();
        for (int d = 1; d < kPlanThreads; d <<= 1) {
            const int a = scan[src][tid] + (tid >= d ? scan[src][tid - d] : 0);
            scan[src ^ 1][tid] = a;
            src ^= 1;
            __syncthreads();
        }
        if (idx < n_bins) off[idx] = carry + scan[src][tid] - v;
        carry += scan[src][kPlanThreads - 1];
        __syncthreads();
    }
    if (tid == 0) off[n_bins] = carry;
    __syncthreads();
    for (int i = tid; i <= n_bins; i += kPlanThreads) p.offsets[i] = off[i];
    // scatter entries to their sorted position (order inside an expert is arbitrary: no result depends on it)
    for (int i = tid; i < n_entries; i += kPlanThreads) {
        const int e = ids[i];
        int pos = -1;
        if (e >= 0 && e < n_experts) {
            pos = off[e] + atomicAdd(&cur[e], 1);
            p.pair_token[pos] = i / top_k;
            p.pair_expert[pos] = e;
        }
        p.pos_of[i] = pos;
    }
    if (with_shared)
        for (int t = tid; t < n_tokens; t += kPlanThreads) {
            p.pair_token[off[n_experts] + t] = t;
            p.pair_expert[off[n_experts] + t] = n_experts;
        }
    // work items: slot s owns sorted pairs [off[s*K], off[(s+1)*K]); the shared expert is slot n_slots
    carry = 0;
    const int n_vslots = n_slots + 1;
    for (int base = 0; base < n_vslots; base += kPlanThreads) {
        const int s = base + tid;
        int lo = 0, hi = 0;
        if (s < n_slots) { lo = off[s * group_size]; hi = off[(s + 1) * group_size]; }
        else if (s == n_slots) { lo = off[n_experts]; hi = off[n_bins]; }
        const int ni = (hi - lo + kPairsPerItem - 1) / kPairsPerItem;
        int src = 0;
        __syncthreads();
        scan[0][tid] = ni;
        __syncthreads();
        for (int d = 1; d < kPlanThreads; d <<= 1) {
            const int a = scan[src][tid] + (tid >= d ? scan[src][tid - d] : 0);
            scan[src ^ 1][tid] = a;
            src ^= 1;
            __syncthreads();
        }
        const int first = carry + scan[src][tid] - ni;
        for (int q = 0; q < ni; ++q) {
            const int it = first + q;
            if (it < p.max_items) {
                p.item_start[it] = lo + q * kPairsPerItem;
                p.item_cnt[it] = min(kPairsPerItem, hi - lo - q * kPairsPerItem);
                p.item_slot[it] = s;
            }
        }
        carry += scan[src][kPlanThreads - 1];
    }
    const int n_items_total = carry;
    // tensor-core work items: expert e (bin n_experts = shared expert) owns sorted pairs [off[e], off[e+1]), cut into
    // blocks of 128 so that one MMA tile never mixes experts
    carry = 0;
    for (int base = 0; base < n_bins; base += kPlanThreads) {
        const int e = base + tid;
        int lo = 0, hi = 0;
        if (e < n_bins) { lo = off[e]; hi = off[e + 1]; }
        const int ni = (hi - lo + kPairsPerGemmItem - 1) / kPairsPerGemmItem;
        int src = 0;
        __syncthreads();
        scan[0][tid] = ni;
        __syncthreads();
        for (int d = 1; d < kPlanThreads; d <<= 1) {
            const int a = scan[src][tid] + (tid >= d ? scan[src][tid - d] : 0);
            scan[src ^ 1][tid] = a;
            src ^= 1;
            __syncthreads();
        }
        const int first = carry + scan[src][tid] - ni;
        for (int q = 0; q < ni; ++q) {
            const int it = first + q;
            if (it < p.max_gitems) {
                p.gitem_start[it] = lo + q * kPairsPerGemmItem;
                p.gitem_cnt[it] = min(kPairsPerGemmItem, hi - lo - q * kPairsPerGemmItem);
                p.gitem_slot[it] = e < n_experts ? e / group_size : n_slots;
            }
        }
        carry += scan[src][kPlanThreads - 1];
    }
    if (tid == 0) {
        p.counters[3] = min(carry, p.max_gitems);
        p.counters[0] = min(n_items_total, p.max_items);
        p.counters[1] = off[n_bins];
        if (reset_status) p.counters[2] = 0;  // otherwise the caller cleared it before the router ran
    }
}

int launch_plan(const chronos_layer_t& L, const int32_t* ids, int n_tokens, int with_shared, const void* x, int x_dtype,
                int reset_status, const Plan& p, cudaStream_t st) {
    plan_kernel<<<1, kPlanThreads, 0, st>>>(ids, n_tokens, L.top_k, L.n_experts, L.group_size, L.n_slots,
                                           with_shared && L.shared_inter > 0, x, x_dtype, L.hidden, reset_status, p);
    return check_launch("plan");
}

}  // namespace chronos
