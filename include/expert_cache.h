/* libexpertcache.so -- C-ABI of the B200 (sm_100a) expert cache.
 *
 * Drop-in for the reference's libexpertcache.so: the same symbol names, argument order,
 * argument meaning and return codes, with cudaStream_t in place of hipStream_t.  Every
 * pointer is device-accessible memory owned by the caller (PyTorch tensors passed as raw
 * pointers; gather sources may be UVA views of pinned host memory).  Every call only
 * enqueues work on `stream`: no host synchronisation and no allocation.  The library keeps
 * per-device kernel attributes and SM counts, looked up on a device's first call.
 *
 * One exception holds device memory of its own: expert_cache_manage_remap_noalloc writes
 * into a library-owned device array, so its first call on each device (which looks up that
 * array's address) must come before any stream capture on that device.
 *
 * Return codes: 0 = enqueued; -1 = arguments refused (nothing enqueued); -2 = E above
 * EXPERT_CACHE_NOALLOC_MAX_EXPERTS (expert_cache_manage_remap_noalloc only); any other
 * value is the cudaError_t of the launch or of a first-call attribute lookup.
 */
#ifndef EXPERT_CACHE_H
#define EXPERT_CACHE_H

#include <cuda_runtime_api.h>

#if defined(__GNUC__)
#define EXPERT_CACHE_API __attribute__((visibility("default")))
#else
#define EXPERT_CACHE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Largest slot count / insert cap per call (reference kernels/expert_cache.hip:80-81). */
#define EXPERT_CACHE_MAX_SLOTS 1024
#define EXPERT_CACHE_MAX_INSERTS 1024
/* Largest expert count.  The reference manage kernel has no bound; this one mirrors the
 * expert->slot table in shared memory, which bounds E (E * 5 bytes + slot state). */
#define EXPERT_CACHE_MAX_EXPERTS 32768
/* Number of (dst, src, bytes) triples one gather call takes (reference _lib.py:61). */
#define EXPERT_CACHE_GATHER_SLOTS 6

/* One policy step for one MoE layer: mark the routed experts, refresh hit priorities
 * (LRU: stamp = step; LFU: stamp + 1, halved every `decay` steps), evict the lowest
 * (stamp, slot) slots whose expert is not routed this step, rewrite table / map_cold /
 * slot_expert / slot_stamp, and emit the (expert, slot) miss list in ascending expert id.
 *
 *   topk_ids     [mk] int32 routed expert ids; < 0 is padding, >= E is ignored
 *   max_distinct more distinct routed experts than this: read-through (only `step` and
 *                `routed` change)
 *   max_inserts  cap on installs this call; `miss` must hold 2*max_inserts ints
 *   table        [E] expert -> slot or -1          map_cold [E] expert -> itself or -1
 *   slot_expert  [S] slot -> expert or -1          slot_stamp [S] int64 priority
 *   routed       [E] uint8 scratch: left holding this step's routed flags
 *   step         [1] int64 call counter            miss [2*max_inserts], n_miss [1]
 *   policy       0 = LRU, 1 = LFU                  decay  LFU halving period, 0 = never
 *
 * Returns -1 if E <= 0, E > EXPERT_CACHE_MAX_EXPERTS, S <= 0, S > EXPERT_CACHE_MAX_SLOTS,
 * max_inserts outside [0, EXPERT_CACHE_MAX_INSERTS] or policy outside {0, 1}; mk <= 0 is
 * an empty step (the counter still advances).
 *
 * Replaces: expert_cache_manage, reference kernels/expert_cache.hip:592-603 (kernel
 * :191-282), bound by vllm_expert_cache/_lib.py:44-47, called from cache.py:118-133. */
EXPERT_CACHE_API int expert_cache_manage(const int* topk_ids, int mk, int E, int S, int max_distinct,
                        int max_inserts, int* table, int* map_cold, int* slot_expert,
                        long long* slot_stamp, unsigned char* routed, long long* step,
                        int* miss, int* n_miss, int policy, int decay,
                        cudaStream_t stream);

/* expert_cache_manage followed, in the same single-CTA launch, by the routing remap
 * out_ids[i] = table[topk_ids[i]] on the updated table (torch indexing semantics: a
 * negative id counts from the end; ids outside [-E, E) give -1).  out_ids holds mk
 * elements of out_elem_bytes (4 = int32, 8 = int64) each.  Returns -1 on the manage
 * rules above, when out_elem_bytes is not 4 or 8, or when out_ids is NULL and mk > 0.
 *
 * Replaces: the torch remap `table[topk_ids.to(int64)].to(topk_ids.dtype)` of reference
 * vllm_expert_cache/cache.py:108-110 that follows the manage call at :118-163.  It has
 * no counterpart symbol in the reference library. */
EXPERT_CACHE_API int expert_cache_manage_remap(const int* topk_ids, int mk, int E, int S, int max_distinct,
                              int max_inserts, int* table, int* map_cold, int* slot_expert,
                              long long* slot_stamp, unsigned char* routed, long long* step,
                              int* miss, int* n_miss, int policy, int decay, void* out_ids,
                              int out_elem_bytes, cudaStream_t stream);

/* expert_cache_manage for an expert-parallel layer, where this rank holds E of the
 * E_global experts.
 *
 * topk_ids are global expert ids. Each is translated on load through
 * expert_map [E_global] (int32: global id -> local expert in [0, E), or -1 for another
 * rank's expert) before the policy sees it. Ids outside [0, E_global) and map entries
 * outside [0, E) count as padding. The policy step is then expert_cache_manage's on the
 * local ids.
 *
 * In the same launch the updated table is composed with the map:
 *   out_map[g] = expert_map[g] in [0, E) ? table[expert_map[g]] : -1   (int32, E_global)
 * This is a global id -> slot map for a kernel that takes an expert map (vLLM's fused
 * MoE with expert_map). The routing ids themselves are left untouched.
 *
 * Returns -1 on the manage rules above, or when expert_map or out_map is NULL, or when
 * E_global <= 0.
 *
 * Has no counterpart in the reference: the reference refuses expert-parallel layers
 * (vllm_expert_cache/backends/generic.py:145-149). It composes the reference's manage
 * step (kernels/expert_cache.hip:191-282) with vLLM's expert map
 * (vllm/model_executor/layers/fused_moe/expert_map_manager.py:22-113). */
EXPERT_CACHE_API int expert_cache_manage_ep(
    const int* topk_ids, int mk, const int* expert_map, int E_global, int E, int S,
    int max_distinct, int max_inserts, int* table, int* map_cold, int* slot_expert,
    long long* slot_stamp, unsigned char* routed, long long* step, int* miss, int* n_miss,
    int policy, int decay, int* out_map, cudaStream_t stream);

/* Install predicted experts ahead of their layer's step (next-layer prefetch).
 *
 * Arguments are expert_cache_manage's without `decay`. pred_ids are the predicted
 * routing. The call installs the missing ones exactly as a manage step would:
 *   - same victim order;
 *   - new slots get priority `step` (LRU) or 1 (LFU);
 *   - miss list and n_miss are written for a following expert_cache_gather.
 *
 * Nothing else changes:
 *   - `step` does not advance;
 *   - hits keep their priority;
 *   - no ageing runs.
 * Slots whose expert is flagged in `routed` on entry are parked like predicted ones, so
 * when the call before this one was the layer's own step, its experts are never evicted.
 * `routed` is left holding the predicted flags.
 *
 * A wrong prediction therefore costs transfers and evictions, never results: the
 * layer's own step still installs whatever it routes.
 *
 * Returns -1 on the manage rules.
 *
 * Has no counterpart in the reference: its README names next-layer prefetch as
 * unexplored (README.md:392-394). */
EXPERT_CACHE_API int expert_cache_prefetch(
    const int* pred_ids, int mk, int E, int S, int max_distinct, int max_inserts, int* table,
    int* map_cold, int* slot_expert, long long* slot_stamp, unsigned char* routed,
    long long* step, int* miss, int* n_miss, int policy, cudaStream_t stream);

/* Limits of expert_cache_pregate. Its shared memory holds one token row and E scores. */
#define EXPERT_CACHE_PREGATE_MAX_HIDDEN 16384
#define EXPERT_CACHE_PREGATE_MAX_EXPERTS 2048

/* Predict a layer's routing from a hidden state.
 *
 * For each of T tokens, out_ids[t*k + r] is the r-th highest score over the E experts,
 * where the score is the dot product of x[t, :H] (bf16, row stride ldx elements) with
 * gate_w[e, :H] (bf16, [E, H] row-major: a router's weight), accumulated in fp32.
 *   - Ties go to the lower expert id.
 *   - NaN scores are never picked.
 *   - Fewer than k finite scores leave -1.
 * Softmax and renormalisation are monotonic, so this is the router's own top-k for the
 * given input. Grouped or biased routers are only approximated. One CTA per token.
 *
 * Returns -1 if:
 *   - T < 0;
 *   - H <= 0, H % 8 != 0 or H > EXPERT_CACHE_PREGATE_MAX_HIDDEN;
 *   - ldx < H or ldx % 8 != 0;
 *   - E <= 0 or E > EXPERT_CACHE_PREGATE_MAX_EXPERTS;
 *   - k outside [1, 32];
 *   - x or gate_w is not 16-byte aligned.
 * T == 0 enqueues nothing.
 *
 * Has no counterpart in the reference. */
EXPERT_CACHE_API int expert_cache_pregate(const void* x, int T, int ldx, int H,
                                          const void* gate_w, int E, int k, int* out_ids,
                                          cudaStream_t stream);

/* Largest expert count of expert_cache_fused (reference expert_cache.hip:341, MAXE). */
#define EXPERT_CACHE_FUSED_MAX_EXPERTS 1024

/* Manage step fused with both of vLLM's moe_align_block_size outputs, in one launch.
 *
 * The manage part is expert_cache_manage with LRU priorities and no ageing (the
 * reference's fused path has no policy argument).  Then, on the updated table, the
 * routing ids are bucketed twice, as moe_align_block_size(topk_ids, bs, ..., map,
 * ignore_invalid_experts=True) would:
 *   hot  side: tokens whose expert is resident, bucket = its SLOT (table[e]);
 *   cold side: the others, bucket = the expert id (map_cold[e]).
 * For each side: sorted_* [L] holds token indices grouped by bucket, each bucket padded
 * to a multiple of bs with the sentinel mk; eids_* [NB] holds the bucket of each block
 * (-1 for unused blocks); npad_* [1] the padded total.  Tokens inside a bucket are in
 * ascending index order for every mk (the reference guarantees that only for mk <= 256).
 * L and NB must be the lengths vLLM's wrapper allocates:
 *   L = mk < E ? min(mk*bs, mk + E*(bs-1)) : mk + E*(bs-1);  NB = ceil(L / bs);
 * writes past L / NB are dropped rather than made.
 *
 * Returns -1 if E <= 0, E > EXPERT_CACHE_FUSED_MAX_EXPERTS, S <= 0,
 * S > EXPERT_CACHE_MAX_SLOTS, bs/L/NB <= 0, mk < 0 or max_inserts outside
 * [0, EXPERT_CACHE_MAX_INSERTS].
 *
 * Replaces: expert_cache_fused, reference kernels/expert_cache.hip:610-624 (kernel
 * :431-588); exported there and checked by kernels/build.sh:36-38, not called by the
 * reference's Python. */
EXPERT_CACHE_API int expert_cache_fused(
    const int* topk_ids, int mk, int E, int S, int max_distinct, int max_inserts, int* table,
    int* map_cold, int* slot_expert, long long* slot_stamp, unsigned char* routed,
    long long* step, int* miss, int* n_miss, int bs, int L, int NB, int* sorted_hot,
    int* eids_hot, int* npad_hot, int* sorted_cold, int* eids_cold, int* npad_cold,
    cudaStream_t stream);

/* Largest expert count accepted by expert_cache_manage_remap_noalloc: the size, in bytes,
 * of the library-owned routed-flag array each GPU holds for it. */
#define EXPERT_CACHE_NOALLOC_MAX_EXPERTS 8192

/* expert_cache_manage_remap for callers that cannot allocate device memory.
 *
 * Some callers cannot call cudaMalloc at all: an engine that has already handed every
 * free byte of HBM to its own pool (a serving stack that sized its KV cache to the card),
 * a host runtime whose device memory comes only from a foreign allocator, or a latency-
 * critical loop where cudaMalloc's implicit device-wide synchronisation is not allowed.
 * The other manage entry points need one caller-allocated scratch array, `routed` (E
 * bytes); this one takes no `routed` argument and writes those flags into a fixed array
 * inside the library instead.  Everything else -- ids, state, miss list, out_ids -- is
 * still passed by the caller, with the same meaning, and the results are identical.
 *
 * Limits and rules:
 *   - E must not exceed EXPERT_CACHE_NOALLOC_MAX_EXPERTS; a larger E returns -2 and
 *     enqueues nothing.  All other argument errors return -1 as for the other entry
 *     points.
 *   - The array is a file-scope device variable: every GPU that loads the library holds
 *     EXPERT_CACHE_NOALLOC_MAX_EXPERTS bytes for it until the process exits.
 *   - The first call on each device looks up the array's device address (once, with that
 *     device current); make that first call before any stream capture begins.
 *   - Every call on a device shares the one array and leaves the last call's flags in
 *     it; each call rewrites entries [0, E) before finishing and nothing has to start at
 *     zero.  Calls that overlap on the GPU (different streams, no ordering between
 *     them) race on the array's contents; the kernel never reads the array back, so
 *     their outputs are unaffected, but the array's contents are then unspecified.
 *   - No cudaMalloc, cudaFree or other allocating call is made.
 *
 * Has no counterpart in the reference: the reference's entry points all take `routed`
 * from the caller. */
EXPERT_CACHE_API int expert_cache_manage_remap_noalloc(
    const int* topk_ids, int mk, int E, int S, int max_distinct, int max_inserts, int* table,
    int* map_cold, int* slot_expert, long long* slot_stamp, long long* step, int* miss,
    int* n_miss, int policy, int decay, void* out_ids, int out_elem_bytes,
    cudaStream_t stream);

/* Copy every installed miss's slabs: for j < *n_miss, e = miss[2j], s = miss[2j+1],
 * dst_k[s*b_k .. (s+1)*b_k) = src_k[e*b_k .. (e+1)*b_k) for the six triples.  Sources are
 * usually UVA views of pinned host memory (the copy then streams over the host link).
 * Identical triples (the caller's padding) are copied once.  chunks * lanes is the CTA
 * budget of the launch (defaults 16 * 64 in the reference's Python layer); the launch
 * uses min(budget, 2 * SM count) CTAs.
 *
 * Returns -1 if any b_k <= 0 or b_k % 16, any dst/src not 16-byte aligned, or
 * chunks <= 0 / lanes <= 0.
 *
 * Replaces: expert_cache_gather, reference kernels/expert_cache.hip:626-643 (kernel
 * :286-314), bound by vllm_expert_cache/_lib.py:50-53, called from cache.py:135-161. */
EXPERT_CACHE_API int expert_cache_gather(void* d0, const void* s0, long b0, void* d1, const void* s1,
                        long b1, void* d2, const void* s2, long b2, void* d3,
                        const void* s3, long b3, void* d4, const void* s4, long b4,
                        void* d5, const void* s5, long b5, const int* miss,
                        const int* n_miss, int chunks, int lanes, cudaStream_t stream);

/* Largest slot count of expert_cache_step: its policy step runs in one CTA of 256 threads,
 * one slot per thread. */
#define EXPERT_CACHE_STEP_MAX_SLOTS 256
/* Wait bound of expert_cache_step when max_wait_us is 0: one second. */
#define EXPERT_CACHE_STEP_DEFAULT_WAIT_US 1000000

/* One whole cached step in a single launch: expert_cache_manage_remap followed by
 * expert_cache_gather of the six triples, with the same arguments, meaning and results.
 *
 * A decode step that installs nothing is then one kernel node instead of two.  Inside the
 * launch, the first CTA to start runs the policy step and the remap and publishes the
 * miss count in a device word tagged with the launch's epoch; the other CTAs wait for
 * that word (bounded by max_wait_us, 0 = EXPERT_CACHE_STEP_DEFAULT_WAIT_US) and then every
 * CTA claims 32 KiB tiles of the slabs' copy until none are left.  The policy CTA copies
 * too, so it completes the copy alone if the others never see the word: a wait that runs
 * out costs time, never bytes.
 *
 *   sync   [8] int32 (8-byte aligned), zero before the first call and then owned by these
 *          calls: [0..1] the arrival word (epoch, CTAs arrived), which the last CTA of a
 *          launch moves to the next epoch, [2..3] the tagged miss-count word, [4] the
 *          current launch's tile counter, [5] a running count of CTAs whose wait ran out,
 *          [6..7] a running int64 count of installed experts (the sum of n_miss over
 *          calls).  Nothing has to be reset between calls, including CUDA-graph replays
 *          of one captured call.  Use one sync array per cache (per layer); launches
 *          sharing one must be ordered on one stream.
 *
 * Returns -1 on the rules of expert_cache_manage_remap and expert_cache_gather, when
 * S > EXPERT_CACHE_STEP_MAX_SLOTS, when sync is NULL or not 8-byte aligned, when
 * max_wait_us < 0, or when max_inserts experts' slabs would be 2^31 or more 32 KiB tiles
 * (64 GiB per expert at max_inserts = 1024).
 *
 * Replaces: the two launches of the reference's per-layer step (cache.py:118-161:
 * expert_cache_manage, kernels/expert_cache.hip:592-603, then expert_cache_gather,
 * :626-643).  It has no counterpart symbol in the reference library; the reference names
 * launch count as the per-layer cost it fused against (expert_cache.hip:316-330). */
EXPERT_CACHE_API int expert_cache_step(
    const int* topk_ids, int mk, int E, int S, int max_distinct, int max_inserts, int* table,
    int* map_cold, int* slot_expert, long long* slot_stamp, unsigned char* routed,
    long long* step, int* miss, int* n_miss, int policy, int decay, void* out_ids,
    int out_elem_bytes, void* d0, const void* s0, long b0, void* d1, const void* s1, long b1,
    void* d2, const void* s2, long b2, void* d3, const void* s3, long b3, void* d4,
    const void* s4, long b4, void* d5, const void* s5, long b5, int chunks, int lanes,
    int* sync, int max_wait_us, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* EXPERT_CACHE_H */
