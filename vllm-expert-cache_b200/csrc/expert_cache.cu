// libexpertcache.so for B200 (sm_100a): the per-layer, per-forward expert-cache hot path.
//
// Two kernels, both launched on the caller's stream with no host synchronisation, so they
// are recorded into vLLM's CUDA graphs like any other node:
//
//   manage_kernel  one CTA.  The whole layer state (E experts, S <= 1024 slots) is read
//                  with one round of coalesced loads into shared memory; the step is then
//                  computed with warp ballots and three or four CTA barriers; results are
//                  written straight back.  Optionally it ends with the routing remap
//                  out_ids[i] = table[topk_ids[i]] on the updated table, so the separate
//                  torch gather/cast kernels of the Python remap disappear.  The
//                  expert-parallel variant instead translates global ids through vLLM's
//                  expert_map on load and ends by writing the composed global id -> slot
//                  map.
//
//   gather_kernel  copies every missing expert's slabs from host memory (UVA views of
//                  pinned pages) into its slot.  The work of all misses and all buffers is
//                  flattened into 32 KiB tiles spread over a fixed grid, so the copy is
//                  balanced whether one expert or eight are missing; each thread keeps
//                  eight 16-byte loads in flight to cover the host-link latency.
//
// Both kernels are Programmatic-Dependent-Launch aware: manage releases its dependents as
// soon as it starts, and gather (launched with programmatic stream serialisation) does
// its set-up before `griddepcontrol.wait`, so its launch latency hides under manage.
//
// Determinism: no atomics and no order-dependent reductions.  Misses are enumerated in
// ascending expert id and victims are ranked by the total order on (stamp, slot), so every
// tensor-parallel rank that sees the same routing evolves the same state.
//
// Semantics follow the reference kernel kernels/expert_cache.hip:191-282 (manage),
// :106-189 (victim choice), :286-314 (gather) and the remap of
// vllm_expert_cache/cache.py:108-110; the C-ABI at the bottom keeps the reference's
// symbols, argument order and return codes (expert_cache.hip:590-645).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <climits>
#include <cstdint>

#include "expert_cache.h"

// Routed-flag array of expert_cache_manage_remap_noalloc, owned by the library so that
// entry point allocates nothing.  Host code must not pass this name to a kernel: on the
// host it is only a stand-in symbol; its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_routed[EXPERT_CACHE_NOALLOC_MAX_EXPERTS];

namespace {

constexpr int kSlotBits = 20;                 // key = stamp << 20 | slot
constexpr long long kParked = LLONG_MAX;      // key of a slot that must not be evicted
constexpr int kMaxDevices = 64;

// ---------------------------------------------------------------------------------------
// PDL helpers (sm_90+).  Without the launch attribute both are no-ops.
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void release_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------------------
// manage

struct ManageArgs {
  const int* ids;
  int mk, E, S, max_distinct, max_inserts;
  int* table;
  int* map_cold;
  int* slot_expert;
  long long* slot_stamp;
  unsigned char* routed;
  long long* step;
  int* miss;
  int* n_miss;
  int policy, decay;
  void* out_ids;        // nullptr: no remap
  int out_elem_bytes;   // 4 or 8
  // Expert parallelism (nullptr / 0 otherwise): routed ids are global and pass through
  // emap [Eg] (global id -> local expert, -1 = another rank's); the launch ends by writing
  // out_map [Eg] = the composed map global id -> slot (-1 = not resident here).
  const int* emap;
  int Eg;
  int* out_map;
  // Prefetch (expert_cache_prefetch): install the predicted experts that are missing and
  // change nothing else -- no step advance, no priority refresh of hits, no ageing -- and
  // never evict a slot whose expert is flagged in `routed` on entry (the previous call's
  // routing: the layer's own step, when prefetches and steps alternate).
  int prefetch;
};

// A routed id as the policy sees it: the id itself or, under expert parallelism, the local
// expert it maps to (-1 for another rank's expert and for ids outside the map).
__device__ __forceinline__ int local_expert(const ManageArgs& a, int id) {
  if (a.emap == nullptr) return id;
  return (id >= 0 && id < a.Eg) ? a.emap[id] : -1;
}

// Dynamic shared memory: key[Spad] i64 | stamp[Spad] i64 | table[E] i32 | slot_expert[S]
// i32 | routed flag[E] u8.  Spad = S rounded up to even so keys can be read in pairs.
__host__ __device__ inline size_t manage_smem_bytes(int E, int S) {
  const size_t spad = (size_t)((S + 1) & ~1);
  return spad * 16 + (size_t)E * 4 + (size_t)S * 4 + (size_t)E;
}

__device__ __forceinline__ void remap_tail(const int* __restrict__ ids, int mk, int E,
                                           void* out, int out_elem_bytes,
                                           const int* s_tab, int my_id, int nt) {
  for (int i = threadIdx.x; i < mk; i += nt) {
    const int id = (i == (int)threadIdx.x) ? my_id : ids[i];
    long long v = -1;
    if (id >= -E && id < E) v = s_tab[id < 0 ? id + E : id];
    if (out_elem_bytes == 8)
      static_cast<long long*>(out)[i] = v;
    else
      static_cast<int*>(out)[i] = (int)v;
  }
}

// Shared-memory views of one manage call (layout: manage_smem_bytes).
struct ManageSmem {
  long long* key;        // [spad] eviction keys
  long long* stamp;      // [spad] priorities after hits / ageing
  int* table;            // [E] expert -> slot, updated by the installs
  int* slot_expert;      // [S]
  unsigned char* flag;   // [E] routed this step
};

__device__ __forceinline__ ManageSmem manage_smem(unsigned char* base, int E, int S) {
  const int spad = (S + 1) & ~1;
  ManageSmem m;
  m.key = reinterpret_cast<long long*>(base);
  m.stamp = m.key + spad;
  m.table = reinterpret_cast<int*>(m.stamp + spad);
  m.slot_expert = m.table + E;
  m.flag = reinterpret_cast<unsigned char*>(m.slot_expert + S);
  return m;
}

// The one round of loads of a policy step: table, routed flags and slot state into shared
// memory (no barrier).  Returns the step counter as read before this call advances it.
// Flag bits: 1 = routed by this call's ids; 2 = routed by the previous step (prefetch
// only: those slots are parked, not installed).
template <int NT>
__device__ __forceinline__ long long manage_stage(const ManageArgs& a, const ManageSmem& sm) {
  const int t = threadIdx.x;
  const long long step0 = a.step[0];
  for (int e = t; e < a.E; e += NT) {
    sm.table[e] = a.table[e];
    sm.flag[e] = (a.prefetch && a.routed[e]) ? 2 : 0;
  }
  for (int s = t; s < a.S; s += NT) {
    sm.slot_expert[s] = a.slot_expert[s];
    sm.stamp[s] = a.slot_stamp[s];
  }
  return step0;
}

// One policy step for the whole CTA (NT threads, S <= NT).  Thread t owns slot t; experts
// are processed in tiles of NT (thread t owns expert base + t), in ascending id.  All
// global state is read once into shared memory and written back directly.  On return
// `sm.table` holds the updated expert->slot table, but only for the installing threads'
// own writes: the caller needs a CTA barrier before reading it when this returns true
// (true = installs happened).  `my_id` is topk_ids[t] (or -1 when t >= mk).  With
// `staged`, manage_stage already ran and a CTA barrier followed it; `step0` is its value.
// `n_out`, when given, receives n_miss in thread 0.
template <int NT>
__device__ __forceinline__ bool manage_core(const ManageArgs& a, const ManageSmem& sm,
                                            int my_id, bool staged = false,
                                            long long step0 = 0, int* n_out = nullptr) {
  constexpr int NW = NT / 32;
  __shared__ int s_missing[EXPERT_CACHE_MAX_INSERTS];   // r-th missing expert, ascending
  __shared__ int w_routed[2][NW], w_missed[2][NW], w_evict[NW];

  const int E = a.E, S = a.S;
  const int spad = (S + 1) & ~1;
  long long* s_key = sm.key;
  long long* s_st = sm.stamp;
  int* s_tab = sm.table;
  int* s_se = sm.slot_expert;
  unsigned char* s_flag = sm.flag;

  const int t = threadIdx.x, lane = t & 31, w = t >> 5;

  // ---- one round of loads: step, table, slot state (ids were read by the caller) -------
  if (!staged) {
    step0 = manage_stage<NT>(a, sm);
    __syncthreads();
  }
  const long long now = step0 + (a.prefetch ? 0 : 1);
  if (t == 0 && !a.prefetch) a.step[0] = now;   // every thread read the old value above

  // ---- routed flags (every writer of an entry stores the same value) -------------------
  if (my_id >= 0 && my_id < E) s_flag[my_id] |= 1;
  for (int i = t + NT; i < a.mk; i += NT) {
    const int e = local_expert(a, a.ids[i]);
    if (e >= 0 && e < E) s_flag[e] |= 1;
  }
  __syncthreads();

  // ---- slot side: parked = holds an expert routed now; hit = refreshed priority --------
  int se = -1;
  bool parked = false, hit = false;
  long long stamp = 0;
  if (t < S) {
    se = s_se[t];
    parked = se >= 0 && se < E && s_flag[se];
    hit = parked && s_tab[se] == t;
    stamp = s_st[t];
    if (hit && !a.prefetch) stamp = (a.policy == 0) ? now : stamp + 1;
  }
  {
    const unsigned b = __ballot_sync(0xffffffffu, t < S && !parked);
    if (lane == 0) w_evict[w] = __popc(b);
  }

  // ---- expert side: distinct count and the ascending miss list --------------------------
  int distinct = 0, n_missing = 0;
  for (int base = 0, tile = 0; base < E; base += NT, ++tile) {
    const int e = base + t;
    const bool f = e < E && (s_flag[e] & 1);
    const bool m = f && s_tab[e] < 0;
    const unsigned bf = __ballot_sync(0xffffffffu, f);
    const unsigned bm = __ballot_sync(0xffffffffu, m);
    const int par = tile & 1;   // double buffer: the next tile's writes never race reads
    if (lane == 0) {
      w_routed[par][w] = __popc(bf);
      w_missed[par][w] = __popc(bm);
    }
    __syncthreads();
    int before = 0, tile_routed = 0, tile_missed = 0;
#pragma unroll
    for (int k = 0; k < NW; ++k) {
      const int c = w_missed[par][k];
      before += (k < w) ? c : 0;
      tile_missed += c;
      tile_routed += w_routed[par][k];
    }
    if (m) {
      const int pos = n_missing + before + __popc(bm & ((1u << lane) - 1u));
      if (pos < EXPERT_CACHE_MAX_INSERTS) s_missing[pos] = e;
    }
    distinct += tile_routed;
    n_missing += tile_missed;
  }
  int n_evict = 0;
#pragma unroll
  for (int k = 0; k < NW; ++k) n_evict += w_evict[k];

  for (int e = t; e < E; e += NT) a.routed[e] = s_flag[e] & 1;

  const bool read_through = distinct > a.max_distinct;
  const int nins = read_through ? 0 : min(n_missing, a.max_inserts);
  if (nins == 0) {
    // Nothing to install: a read-through step changes no priority; otherwise the hits
    // keep their refreshed priority and no ageing runs (it only runs on inserting steps).
    if (!read_through && hit) a.slot_stamp[t] = stamp;
    if (t == 0) a.n_miss[0] = 0;
    if (t == 0 && n_out) *n_out = 0;
    return false;
  }

  // ---- ageing, eviction keys, miss list -------------------------------------------------
  const bool age = !a.prefetch && a.policy != 0 && a.decay > 0 &&
                   (now % (long long)a.decay) == 0;
  if (t < S) {
    if (age) stamp >>= 1;
    s_st[t] = stamp;
    s_key[t] = parked ? kParked : ((stamp << kSlotBits) | (long long)t);
  }
  if (t == 0 && (S & 1)) s_key[S] = kParked;
  for (int j = t; j < nins; j += NT) a.miss[2 * j] = s_missing[j];
  __syncthreads();

  // ---- rank every slot's key: G lanes per slot, pairs of keys per 16-byte load ----------
  int G = 1;
  while (G < 32 && 2 * G * S <= NT) G <<= 1;
  const int slot = t / G, q = t & (G - 1);
  long long key = kParked;
  int rank = 0;
  if (slot < S) {
    key = s_key[slot];
    const longlong2* kp = reinterpret_cast<const longlong2*>(s_key);
    for (int p = q; p < (spad >> 1); p += G) {
      const longlong2 v = kp[p];
      rank += (v.x < key) + (v.y < key);
    }
  }
  for (int off = G >> 1; off; off >>= 1) rank += __shfl_xor_sync(0xffffffffu, rank, off);

  // ---- install: the r-th smallest evictable key takes the r-th missing expert -----------
  const long long fresh = (a.policy == 0) ? now : 1;
  if (q == 0 && slot < S) {
    if (key != kParked && rank < nins) {
      const int e = s_missing[rank];
      const int old = s_se[slot];
      if (old >= 0 && old < E) {
        a.table[old] = -1;
        a.map_cold[old] = old;
        s_tab[old] = -1;
      }
      a.table[e] = slot;
      a.map_cold[e] = -1;
      s_tab[e] = slot;
      a.miss[2 * rank + 1] = slot;
      a.slot_expert[slot] = e;
      a.slot_stamp[slot] = fresh;
    } else {
      a.slot_stamp[slot] = s_st[slot];
    }
  }
  if (t == 0) a.n_miss[0] = min(nins, n_evict);
  if (t == 0 && n_out) *n_out = min(nins, n_evict);
  return true;
}

// expert_cache_manage / _manage_remap / _manage_ep: the policy step, then (optionally)
// the remap of the routing ids, or the composed expert-parallel map, on the updated table.
template <int NT>
__global__ void __launch_bounds__(NT, 1) manage_kernel(const __grid_constant__ ManageArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const ManageSmem sm = manage_smem(smem, a.E, a.S);
  grid_dependency_wait();     // topk_ids may come from the kernel just before us
  release_dependents();       // let the gather launch and park on its own wait
  const int t = threadIdx.x;
  const int my_id = (t < a.mk) ? local_expert(a, a.ids[t]) : -1;
  const bool changed = manage_core<NT>(a, sm, my_id);
  if (a.out_ids) {            // never set together with emap (host rule)
    if (changed) __syncthreads();
    remap_tail(a.ids, a.mk, a.E, a.out_ids, a.out_elem_bytes, sm.table, my_id, NT);
  }
  if (a.out_map) {
    if (changed) __syncthreads();
    for (int g = t; g < a.Eg; g += NT) {
      const int e = a.emap[g];
      a.out_map[g] = (e >= 0 && e < a.E) ? sm.table[e] : -1;
    }
  }
}

// ---------------------------------------------------------------------------------------
// fused: manage + both moe_align_block_size outputs (reference expert_cache.hip:316-588)

struct AlignArgs {
  int bs, L, NB;
  int* sorted_hot;
  int* eids_hot;
  int* npad_hot;
  int* sorted_cold;
  int* eids_cold;
  int* npad_cold;
};

// Extra dynamic shared memory after the manage layout: cnt_h[S] cum_h[S+1] cnt_c[E]
// cum_c[E+1] (ints).
__host__ __device__ inline size_t fused_smem_bytes(int E, int S) {
  return manage_smem_bytes(E, S) + (size_t)(2 * S + 2 * E + 2) * 4 + 16;
}

// Exclusive scan of one value per thread across the CTA; *total gets the CTA sum.  The
// caller separates two uses of `warp_buf` with a barrier.
template <int NT>
__device__ __forceinline__ int cta_exclusive_scan(int v, int* warp_buf, int* total) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_buf[w] = x;
  __syncthreads();
  int before = 0, sum = 0;
#pragma unroll
  for (int k = 0; k < NW; ++k) {
    const int c = warp_buf[k];
    before += (k < w) ? c : 0;
    sum += c;
  }
  *total = sum;
  return before + x - v;
}

// cum[b] = sum over j < b of roundup(cnt[j], bs); cum[n] = total.  Thread t owns the
// contiguous buckets [t*C, t*C + C).
template <int NT>
__device__ __forceinline__ void padded_scan(const int* cnt, int* cum, int n, int bs,
                                            int* warp_buf) {
  const int C = (n + NT - 1) / NT;
  const int lo = threadIdx.x * C, hi = min(lo + C, n);
  int mine = 0;
  for (int b = lo; b < hi; ++b) mine += (cnt[b] + bs - 1) / bs * bs;
  int total = 0;
  int run = cta_exclusive_scan<NT>(mine, warp_buf, &total);
  for (int b = lo; b < hi; ++b) {
    cum[b] = run;
    run += (cnt[b] + bs - 1) / bs * bs;
  }
  if (threadIdx.x == 0) cum[n] = total;
}

template <int NT>
__global__ void __launch_bounds__(NT, 1)
    fused_kernel(const __grid_constant__ ManageArgs a, const __grid_constant__ AlignArgs g) {
  constexpr int NW = NT / 32;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int warp_h[NW], warp_c[NW];
  const int E = a.E, S = a.S, mk = a.mk;
  const ManageSmem sm = manage_smem(smem, E, S);
  int* cnt_h = reinterpret_cast<int*>(smem + manage_smem_bytes(E, S) + 16 -
                                      (manage_smem_bytes(E, S) & 15));
  int* cum_h = cnt_h + S;
  int* cnt_c = cum_h + S + 1;
  int* cum_c = cnt_c + E;
  const int t = threadIdx.x, lane = t & 31;

  grid_dependency_wait();
  release_dependents();
  const int my_id = (t < mk) ? a.ids[t] : -1;
  manage_core<NT>(a, sm, my_id);   // LRU semantics: the launcher passes policy 0

  // ---- sentinels, cleared counts ---------------------------------------------------------
  for (int i = t; i < g.L; i += NT) {
    g.sorted_hot[i] = mk;
    g.sorted_cold[i] = mk;
  }
  for (int i = t; i < g.NB; i += NT) {
    g.eids_hot[i] = -1;
    g.eids_cold[i] = -1;
  }
  for (int b = t; b < S; b += NT) cnt_h[b] = 0;
  for (int b = t; b < E; b += NT) cnt_c[b] = 0;
  __syncthreads();   // also publishes the installs' table updates

  // ---- one counting pass feeds both sides: resident -> slot bucket, else expert bucket --
  for (int i = t; i < mk; i += NT) {
    const int e = (i == t) ? my_id : a.ids[i];
    if (e < 0 || e >= E) continue;
    const int s = sm.table[e];
    if ((unsigned)s < (unsigned)S)
      atomicAdd(&cnt_h[s], 1);      // integer counts: the result is order-independent
    else
      atomicAdd(&cnt_c[e], 1);
  }
  __syncthreads();
  padded_scan<NT>(cnt_h, cum_h, S, g.bs, warp_h);
  padded_scan<NT>(cnt_c, cum_c, E, g.bs, warp_c);
  __syncthreads();
  if (t == 0) {
    g.npad_hot[0] = cum_h[S];
    g.npad_cold[0] = cum_c[E];
  }

  // ---- block -> bucket ids (the hot side carries slot indices) ---------------------------
  for (int b = t; b < S; b += NT)
    for (int i = cum_h[b]; i < cum_h[b + 1]; i += g.bs)
      if (i / g.bs < g.NB) g.eids_hot[i / g.bs] = b;
  for (int b = t; b < E; b += NT)
    for (int i = cum_c[b]; i < cum_c[b + 1]; i += g.bs)
      if (i / g.bs < g.NB) g.eids_cold[i / g.bs] = b;
  for (int b = t; b < S; b += NT) cnt_h[b] = cum_h[b];   // counts become cursors
  for (int b = t; b < E; b += NT) cnt_c[b] = cum_c[b];
  __syncthreads();

  // ---- placement: one warp walks the tokens in order, so each bucket lists its tokens in
  // ascending index for every mk (match_any ranks lanes that share a bucket) -------------
  if (t < 32) {
    const unsigned below = (1u << lane) - 1u;
    for (int base = 0; base < mk; base += 32) {
      const int i = base + lane;
      int key = -1;
      if (i < mk) {
        const int e = a.ids[i];
        if (e >= 0 && e < E) {
          const int s = sm.table[e];
          key = ((unsigned)s < (unsigned)S) ? s : S + e;
        }
      }
      const unsigned same = __match_any_sync(0xffffffffu, key);
      int* cursor = key < 0 ? nullptr : (key < S ? &cnt_h[key] : &cnt_c[key - S]);
      const int pos = cursor ? *cursor + __popc(same & below) : 0;
      __syncwarp();
      if (cursor && (same & below) == 0) *cursor += __popc(same);
      __syncwarp();
      if (cursor && pos < g.L) (key < S ? g.sorted_hot : g.sorted_cold)[pos] = i;
    }
  }
}

// ---------------------------------------------------------------------------------------
// gather

constexpr int kGatherThreads = 256;
constexpr int kGatherCtasPerSm = 2;
constexpr int kGatherUnroll = 8;                                 // 16-byte loads in flight
constexpr int kTileVecs = kGatherThreads * kGatherUnroll;        // 32 KiB per tile

struct GatherArgs {
  uint4* dst[EXPERT_CACHE_GATHER_SLOTS];
  const uint4* src[EXPERT_CACHE_GATHER_SLOTS];
  long long vecs[EXPERT_CACHE_GATHER_SLOTS];          // 16-byte vectors per expert
  int tile_start[EXPERT_CACHE_GATHER_SLOTS + 1];      // prefix of tiles per expert
  int nbuf;
  const int* miss;
  const int* n_miss;
};

__device__ __forceinline__ uint4 load_stream(const uint4* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}

// Copy tiles u = first, first + stride, ... of the flattened work of `nm` misses.  With
// kCoherent the miss list is read from L2 (it was written earlier in the same launch);
// otherwise a previous launch wrote it and plain loads are fine.
template <bool kCoherent>
__device__ __forceinline__ void gather_tiles(const GatherArgs& a, int nm, long long first_u,
                                             long long stride) {
  const int per_miss = a.tile_start[a.nbuf];
  const long long total = (long long)nm * per_miss;
  for (long long u = first_u; u < total; u += stride) {
    const int j = (int)(u / per_miss);
    const int v = (int)(u - (long long)j * per_miss);
    int k = 0;
    while (v >= a.tile_start[k + 1]) ++k;
    const long long first = (long long)(v - a.tile_start[k]) * kTileVecs;
    const long long left = a.vecs[k] - first;
    const long long e = kCoherent ? __ldcg(a.miss + 2 * j) : a.miss[2 * j];
    const long long s = kCoherent ? __ldcg(a.miss + 2 * j + 1) : a.miss[2 * j + 1];
    const uint4* src = a.src[k] + e * a.vecs[k] + first;
    uint4* dst = a.dst[k] + s * a.vecs[k] + first;
    uint4 r[kGatherUnroll];
#pragma unroll
    for (int i = 0; i < kGatherUnroll; ++i) {
      const int x = threadIdx.x + i * kGatherThreads;
      if (x < left) r[i] = load_stream(src + x);
    }
#pragma unroll
    for (int i = 0; i < kGatherUnroll; ++i) {
      const int x = threadIdx.x + i * kGatherThreads;
      if (x < left) dst[x] = r[i];
    }
  }
}

__global__ void __launch_bounds__(kGatherThreads)
    gather_kernel(const __grid_constant__ GatherArgs a) {
  grid_dependency_wait();   // the miss list is written by the manage launch before us
  gather_tiles<false>(a, a.n_miss[0], blockIdx.x, gridDim.x);
}

// ---------------------------------------------------------------------------------------
// step: manage + remap + gather in one launch (expert_cache_step)
//
// A decode step that installs nothing is then one graph node instead of two.  A launch
// tells its own words from a previous launch's by an epoch kept in the arrival word
// (high 32 bits: epoch, low 32 bits: CTAs arrived in this epoch):
//
//   - election: every CTA adds 1 to the arrival word and gets (epoch, ticket).  Ticket 0
//     arrived first -- it is running -- and runs the policy step and the remap.  The CTA
//     that draws ticket G - 1 arrived last; it moves the word to (epoch + 1, 0), so the
//     next launch (or graph replay) starts a new epoch with every counter of this one
//     behind it.  Nothing waits for that: every CTA of this launch already holds its
//     ticket.
//   - publication: the policy CTA resets the tile counter, then publishes
//     ((epoch + 1) << 20 | n_miss) in one release store; the other CTAs wait for a word
//     with their epoch (bounded).
//   - copy: every CTA claims 32 KiB tiles of the miss list's copy from the tile counter
//     until none are left.  The policy CTA claims tiles too, so it alone completes the
//     copy if no other CTA ever sees the word: a wait that runs out (counted, never
//     silent) costs time, never bytes.  For the same reason a helper whose staged table
//     already holds every routed expert leaves without waiting.
// While thread 0 takes its ticket, every thread already stages the state into shared
// memory (small E only), so the ticket's round trip overlaps the state load.
//
// sync (int32[8], 8-byte aligned, zero before first use): [0..1] arrival word (u64),
// [2..3] ready word (u64), [4] tile counter of the current launch, [5] running count of
// waits that ran out, [6..7] running install count (u64).

constexpr int kStepThreads = kGatherThreads;
constexpr int kStepStageMaxExperts = 4096;   // stage speculatively up to this E
constexpr int kReadyShift = 20;              // n_miss <= 1024 < 2^20

struct StepArgs {
  ManageArgs m;
  GatherArgs g;
  int* sync;
  long long wait_ns;       // bound on a CTA's wait for the policy step
  int chunks, lanes;       // CTA budget (host side only)
};

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned long long load_acquire_gpu(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void store_relaxed_gpu(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ void store_release_gpu(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ void copy_tile(const GatherArgs& a, int per_miss, long long u) {
  const int j = (int)(u / per_miss);
  const int v = (int)(u - (long long)j * per_miss);
  int k = 0;
  while (v >= a.tile_start[k + 1]) ++k;
  const long long first = (long long)(v - a.tile_start[k]) * kTileVecs;
  const long long left = a.vecs[k] - first;
  const long long e = __ldcg(a.miss + 2 * j), s = __ldcg(a.miss + 2 * j + 1);
  const uint4* src = a.src[k] + e * a.vecs[k] + first;
  uint4* dst = a.dst[k] + s * a.vecs[k] + first;
  uint4 r[kGatherUnroll];
#pragma unroll
  for (int i = 0; i < kGatherUnroll; ++i) {
    const int x = threadIdx.x + i * kGatherThreads;
    if (x < left) r[i] = load_stream(src + x);
  }
#pragma unroll
  for (int i = 0; i < kGatherUnroll; ++i) {
    const int x = threadIdx.x + i * kGatherThreads;
    if (x < left) dst[x] = r[i];
  }
}

__global__ void __launch_bounds__(kStepThreads, 2) step_kernel(const __grid_constant__ StepArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ unsigned long long s_arrival;
  __shared__ int s_nm, s_tile;
  const int t = threadIdx.x;
  unsigned long long* arrival = reinterpret_cast<unsigned long long*>(a.sync);
  unsigned long long* ready = arrival + 1;
  int* tile_ctr = a.sync + 4;
  grid_dependency_wait();     // ids, state and the previous launch's words are final
  if (t == 0) {
    const unsigned long long v = atomicAdd(arrival, 1ull);
    s_arrival = v;
    if ((unsigned)(v & 0xffffffffu) == gridDim.x - 1)   // the last to arrive: next epoch
      atomicExch(arrival, ((v >> 32) + 1) << 32);
  }
  const ManageSmem sm = manage_smem(smem, a.m.E, a.m.S);
  const int my_id = (t < a.m.mk) ? a.m.ids[t] : -1;
  const bool staged = a.m.E <= kStepStageMaxExperts;
  long long step0 = 0;
  if (staged) step0 = manage_stage<kStepThreads>(a.m, sm);   // overlaps the ticket
  __syncthreads();
  // epoch + 1: the ready word's initial zero never matches
  const unsigned long long tag = ((s_arrival >> 32) + 1) & ((1ull << (64 - kReadyShift)) - 1);
  int nm = 0;
  if ((s_arrival & 0xffffffffu) == 0) {
    manage_core<kStepThreads>(a.m, sm, my_id, staged, step0, &s_nm);
    if (t == 0 && s_nm > 0) *tile_ctr = 0;   // this launch's tiles start at 0
    __syncthreads();                    // installs, miss list, n_miss and table complete
    nm = s_nm;
    if (t == 0) {
      const unsigned long long word = (tag << kReadyShift) | (unsigned long long)nm;
      // Nothing to copy: the other CTAs only need the word itself, so it goes out without
      // the release fence (which would first wait for this CTA's state stores).
      if (nm == 0)
        store_relaxed_gpu(ready, word);
      else
        store_release_gpu(ready, word);
    }
    if (a.m.out_ids)
      remap_tail(a.m.ids, a.m.mk, a.m.E, a.m.out_ids, a.m.out_elem_bytes, sm.table, my_id,
                 kStepThreads);
    // running install count: only the policy CTA writes it, launches are stream-ordered;
    // a step without installs skips the read-modify-write (a memory round trip at the end
    // of the launch)
    if (t == 0 && nm > 0) *reinterpret_cast<long long*>(a.sync + 6) += nm;
  } else {
    if (staged) {
      // A helper that sees every routed expert already in a slot leaves at once.  Its view
      // may be the table before or after the policy CTA's installs, or a mix of the two;
      // either way leaving only forgoes helping: the policy CTA claims whatever tiles
      // are left.  A step that installs nothing never changes the table, so every helper
      // of such a step sees it exactly and none of them waits.
      bool missing = my_id >= 0 && my_id < a.m.E && sm.table[my_id] < 0;
      for (int i = t + kStepThreads; i < a.m.mk; i += kStepThreads) {
        const int e = a.m.ids[i];
        missing |= e >= 0 && e < a.m.E && sm.table[e] < 0;
      }
      if (!__syncthreads_or(missing)) return;
    }
    if (t == 0) {
      const unsigned long long t0 = global_ns();
      unsigned ns = 32;
      int got = -1;
      for (long long it = 0; it < (1LL << 26); ++it) {
        const unsigned long long v = load_acquire_gpu(ready);
        if ((v >> kReadyShift) == tag) {
          got = (int)(v & ((1ull << kReadyShift) - 1));
          break;
        }
        if ((long long)(global_ns() - t0) > a.wait_ns) break;
        __nanosleep(ns);
        if (ns < 128) ns <<= 1;
      }
      if (got < 0) atomicAdd(a.sync + 5, 1);
      s_nm = got < 0 ? 0 : got;
    }
    __syncthreads();
    nm = s_nm;
  }
  if (nm == 0) return;
  const int per_miss = a.g.tile_start[a.g.nbuf];
  const long long total = (long long)nm * per_miss;
  for (;;) {
    if (t == 0) s_tile = atomicAdd(tile_ctr, 1);
    __syncthreads();
    const long long u = s_tile;
    __syncthreads();
    if (u >= total) break;
    copy_tile(a.g, per_miss, u);
  }
}

// ---------------------------------------------------------------------------------------
// pregate: the next layer's routing predicted from this layer's MoE input

constexpr int kPregateThreads = 256;

// One CTA per token.  The token's row is staged in shared memory; each warp scores whole
// experts (16-byte loads of the gate row, fp32 accumulation, a fixed xor-shuffle order),
// then k rounds of a CTA argmax pick the top k (ties -> lower expert id; NaN never wins;
// fewer than k finite scores leave -1).
__global__ void __launch_bounds__(kPregateThreads)
    pregate_kernel(const __nv_bfloat16* __restrict__ x, int ldx, int H,
                   const __nv_bfloat16* __restrict__ w, int E, int k, int* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char smem[];
  uint4* xs = reinterpret_cast<uint4*>(smem);                                  // [H/8]
  float* logit = reinterpret_cast<float*>(smem + (size_t)H * 2);                // [E]
  __shared__ float r_val[kPregateThreads / 32];
  __shared__ int r_idx[kPregateThreads / 32];
  constexpr int NW = kPregateThreads / 32;
  const int tok = blockIdx.x, t = threadIdx.x, lane = t & 31, wp = t >> 5;
  const int hv = H >> 3;

  grid_dependency_wait();
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)tok * ldx);
  for (int i = t; i < hv; i += kPregateThreads) xs[i] = xr[i];
  __syncthreads();

  for (int e = wp; e < E; e += NW) {
    const uint4* wr = reinterpret_cast<const uint4*>(w + (size_t)e * H);
    float acc = 0.f;
    for (int i = lane; i < hv; i += 32) {
      const uint4 a = xs[i];
      const uint4 b = wr[i];
      const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&a);
      const __nv_bfloat162* pb = reinterpret_cast<const __nv_bfloat162*>(&b);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 fa = __bfloat1622float2(pa[j]);
        const float2 fb = __bfloat1622float2(pb[j]);
        acc = fmaf(fa.x, fb.x, acc);
        acc = fmaf(fa.y, fb.y, acc);
      }
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) logit[e] = acc;
  }
  __syncthreads();

  for (int r = 0; r < k; ++r) {
    float bv = -INFINITY;
    int bi = -1;
    for (int e = t; e < E; e += kPregateThreads) {
      const float v = logit[e];
      if (v > bv) { bv = v; bi = e; }        // ascending e: the first of equals stays
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
    }
    if (lane == 0) { r_val[wp] = bv; r_idx[wp] = bi; }
    __syncthreads();
    if (t == 0) {
      float v = -INFINITY;
      int b = -1;
      for (int q = 0; q < NW; ++q)
        if (r_idx[q] >= 0 && (b < 0 || r_val[q] > v || (r_val[q] == v && r_idx[q] < b))) {
          v = r_val[q];
          b = r_idx[q];
        }
      out[(size_t)tok * k + r] = b;
      if (b >= 0) logit[b] = -INFINITY;       // taken: never picked again
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------------------
// host side

int current_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= kMaxDevices) return -1;
  return d;
}

// Opt a kernel into the full shared-memory carve-out once per device (`done` is the
// kernel's own per-device flag array).
template <typename Kernel>
cudaError_t ensure_smem_optin(Kernel fn, std::atomic<bool>* done, int dev) {
  if (done[dev].load(std::memory_order_acquire)) return cudaSuccess;
  int optin = 0;
  cudaError_t err = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (err != cudaSuccess) return err;
  cudaFuncAttributes fa{};
  err = cudaFuncGetAttributes(&fa, fn);
  if (err != cudaSuccess) return err;
  err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             optin - (int)fa.sharedSizeBytes);
  if (err == cudaSuccess) done[dev].store(true, std::memory_order_release);
  return err;
}

template <int NT>
cudaError_t ensure_manage_smem(int dev) {
  static std::atomic<bool> done[kMaxDevices];
  return ensure_smem_optin(manage_kernel<NT>, done, dev);
}

template <int NT>
int launch_manage(const ManageArgs& a, cudaStream_t stream) {
  const size_t smem = manage_smem_bytes(a.E, a.S);
  if (smem > 48 * 1024) {
    const int dev = current_device();
    if (dev < 0) return (int)cudaErrorInvalidDevice;
    const cudaError_t err = ensure_manage_smem<NT>(dev);
    if (err != cudaSuccess) return (int)err;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return (int)cudaLaunchKernelEx(&cfg, manage_kernel<NT>, a);
}

template <int NT>
int launch_fused(const ManageArgs& a, const AlignArgs& g, cudaStream_t stream) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = fused_smem_bytes(a.E, a.S);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return (int)cudaLaunchKernelEx(&cfg, fused_kernel<NT>, a, g);
}

bool manage_args_ok(const ManageArgs& a) {
  if (a.E <= 0 || a.E > EXPERT_CACHE_MAX_EXPERTS) return false;
  if (a.S <= 0 || a.S > EXPERT_CACHE_MAX_SLOTS || a.S > (1 << kSlotBits) - 1) return false;
  if (a.max_inserts < 0 || a.max_inserts > EXPERT_CACHE_MAX_INSERTS) return false;
  return a.policy == 0 || a.policy == 1;
}

int manage_checked(const ManageArgs& a, cudaStream_t stream) {
  if (!manage_args_ok(a)) return -1;
  if (a.S <= 128) return launch_manage<128>(a, stream);
  if (a.S <= 256) return launch_manage<256>(a, stream);
  return launch_manage<1024>(a, stream);
}

ManageArgs make_manage_args(const int* topk_ids, int mk, int E, int S, int max_distinct,
                            int max_inserts, int* table, int* map_cold, int* slot_expert,
                            long long* slot_stamp, unsigned char* routed, long long* step,
                            int* miss, int* n_miss, int policy, int decay) {
  ManageArgs a{};
  a.ids = topk_ids;
  a.mk = mk < 0 ? 0 : mk;
  a.E = E;
  a.S = S;
  a.max_distinct = max_distinct;
  a.max_inserts = max_inserts;
  a.table = table;
  a.map_cold = map_cold;
  a.slot_expert = slot_expert;
  a.slot_stamp = slot_stamp;
  a.routed = routed;
  a.step = step;
  a.miss = miss;
  a.n_miss = n_miss;
  a.policy = policy;
  a.decay = decay;
  a.out_ids = nullptr;
  a.out_elem_bytes = 4;
  a.emap = nullptr;
  a.Eg = 0;
  a.out_map = nullptr;
  a.prefetch = 0;
  return a;
}

// SM count per device, looked up once (sizes the gather grid).
std::atomic<int> g_sm_count[kMaxDevices];

// The six (dst, src, bytes) triples of one gather as kernel arguments: -1 on a refused
// triple.  A triple repeated from an earlier one (the caller's padding) is copied once.
int make_gather_args(void* const* dsts, const void* const* srcs, const long* bytes,
                     const int* miss, const int* n_miss, GatherArgs* out) {
  for (int i = 0; i < EXPERT_CACHE_GATHER_SLOTS; ++i) {
    if (bytes[i] <= 0 || bytes[i] % 16) return -1;
    if ((reinterpret_cast<uintptr_t>(dsts[i]) | reinterpret_cast<uintptr_t>(srcs[i])) & 15)
      return -1;
  }
  GatherArgs a{};
  int n = 0;
  long long tiles = 0;
  a.tile_start[0] = 0;
  for (int i = 0; i < EXPERT_CACHE_GATHER_SLOTS; ++i) {
    bool repeat = false;
    for (int k = 0; k < i; ++k)
      repeat |= dsts[k] == dsts[i] && srcs[k] == srcs[i] && bytes[k] == bytes[i];
    if (repeat) continue;
    a.dst[n] = static_cast<uint4*>(dsts[i]);
    a.src[n] = static_cast<const uint4*>(srcs[i]);
    a.vecs[n] = bytes[i] / 16;
    tiles += (a.vecs[n] + kTileVecs - 1) / kTileVecs;
    if (tiles > INT_MAX / 2) return -1;
    a.tile_start[n + 1] = (int)tiles;
    ++n;
  }
  a.nbuf = n;
  a.miss = miss;
  a.n_miss = n_miss;
  *out = a;
  return 0;
}

// chunks * lanes is the CTA budget; more than two CTAs per SM never moved bytes faster
// (the host link is the bound), and an idle launch (no misses) retires sooner small.
int gather_grid(int chunks, int lanes, unsigned* grid) {
  if (chunks <= 0 || lanes <= 0) return -1;
  const int dev = current_device();
  if (dev < 0) return (int)cudaErrorInvalidDevice;
  int sms = g_sm_count[dev].load(std::memory_order_relaxed);
  if (sms == 0) {
    const cudaError_t err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (err != cudaSuccess) return (int)err;
    g_sm_count[dev].store(sms, std::memory_order_relaxed);
  }
  const long long budget = (long long)chunks * (long long)lanes;
  const long long cap = (long long)kGatherCtasPerSm * sms;
  *grid = (unsigned)(budget < cap ? budget : cap);
  return 0;
}

int launch_step(const StepArgs& a, cudaStream_t stream) {
  const size_t smem = manage_smem_bytes(a.m.E, a.m.S);
  if (smem > 48 * 1024) {
    static std::atomic<bool> done[kMaxDevices];
    const int dev = current_device();
    if (dev < 0) return (int)cudaErrorInvalidDevice;
    const cudaError_t err = ensure_smem_optin(step_kernel, done, dev);
    if (err != cudaSuccess) return (int)err;
  }
  unsigned grid = 0;
  const int rc = gather_grid(a.chunks, a.lanes, &grid);
  if (rc != 0) return rc;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kStepThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return (int)cudaLaunchKernelEx(&cfg, step_kernel, a);
}

// Device address of g_noalloc_routed on the current device, looked up once per device.
std::atomic<void*> g_noalloc_routed_addr[kMaxDevices];

int noalloc_routed_address(void** out) {
  const int dev = current_device();
  if (dev < 0) return (int)cudaErrorInvalidDevice;
  void* p = g_noalloc_routed_addr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_routed);
    if (err != cudaSuccess) return (int)err;
    g_noalloc_routed_addr[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return 0;
}

}  // namespace

extern "C" {

int expert_cache_manage(const int* topk_ids, int mk, int E, int S, int max_distinct,
                        int max_inserts, int* table, int* map_cold, int* slot_expert,
                        long long* slot_stamp, unsigned char* routed, long long* step,
                        int* miss, int* n_miss, int policy, int decay,
                        cudaStream_t stream) {
  const ManageArgs a = make_manage_args(topk_ids, mk, E, S, max_distinct, max_inserts, table,
                                        map_cold, slot_expert, slot_stamp, routed, step,
                                        miss, n_miss, policy, decay);
  return manage_checked(a, stream);
}

int expert_cache_manage_remap(const int* topk_ids, int mk, int E, int S, int max_distinct,
                              int max_inserts, int* table, int* map_cold, int* slot_expert,
                              long long* slot_stamp, unsigned char* routed, long long* step,
                              int* miss, int* n_miss, int policy, int decay, void* out_ids,
                              int out_elem_bytes, cudaStream_t stream) {
  if ((out_ids == nullptr && mk > 0) || (out_elem_bytes != 4 && out_elem_bytes != 8))
    return -1;
  ManageArgs a = make_manage_args(topk_ids, mk, E, S, max_distinct, max_inserts, table,
                                  map_cold, slot_expert, slot_stamp, routed, step, miss,
                                  n_miss, policy, decay);
  a.out_ids = mk > 0 ? out_ids : nullptr;   // nothing to remap: behaves as manage
  a.out_elem_bytes = out_elem_bytes;
  return manage_checked(a, stream);
}

int expert_cache_fused(const int* topk_ids, int mk, int E, int S, int max_distinct,
                       int max_inserts, int* table, int* map_cold, int* slot_expert,
                       long long* slot_stamp, unsigned char* routed, long long* step,
                       int* miss, int* n_miss, int bs, int L, int NB, int* sorted_hot,
                       int* eids_hot, int* npad_hot, int* sorted_cold, int* eids_cold,
                       int* npad_cold, cudaStream_t stream) {
  if (E <= 0 || E > EXPERT_CACHE_FUSED_MAX_EXPERTS || S <= 0 || S > EXPERT_CACHE_MAX_SLOTS)
    return -1;
  if (bs <= 0 || L <= 0 || NB <= 0 || mk < 0) return -1;
  if (max_inserts < 0 || max_inserts > EXPERT_CACHE_MAX_INSERTS) return -1;
  // The fused path is LRU without ageing, like the reference's (expert_cache.hip:481, 505).
  const ManageArgs a = make_manage_args(topk_ids, mk, E, S, max_distinct, max_inserts, table,
                                        map_cold, slot_expert, slot_stamp, routed, step,
                                        miss, n_miss, 0, 0);
  AlignArgs g{};
  g.bs = bs;
  g.L = L;
  g.NB = NB;
  g.sorted_hot = sorted_hot;
  g.eids_hot = eids_hot;
  g.npad_hot = npad_hot;
  g.sorted_cold = sorted_cold;
  g.eids_cold = eids_cold;
  g.npad_cold = npad_cold;
  if (S <= 256) return launch_fused<256>(a, g, stream);
  return launch_fused<1024>(a, g, stream);
}

int expert_cache_manage_remap_noalloc(const int* topk_ids, int mk, int E, int S,
                                      int max_distinct, int max_inserts, int* table,
                                      int* map_cold, int* slot_expert, long long* slot_stamp,
                                      long long* step, int* miss, int* n_miss, int policy,
                                      int decay, void* out_ids, int out_elem_bytes,
                                      cudaStream_t stream) {
  if (E <= 0) return -1;
  if (E > EXPERT_CACHE_NOALLOC_MAX_EXPERTS) return -2;   // beyond the library's array
  void* routed = nullptr;
  const int rc = noalloc_routed_address(&routed);
  if (rc != 0) return rc;
  return expert_cache_manage_remap(topk_ids, mk, E, S, max_distinct, max_inserts, table,
                                   map_cold, slot_expert, slot_stamp,
                                   static_cast<unsigned char*>(routed), step, miss, n_miss,
                                   policy, decay, out_ids, out_elem_bytes, stream);
}

int expert_cache_step(const int* topk_ids, int mk, int E, int S, int max_distinct,
                      int max_inserts, int* table, int* map_cold, int* slot_expert,
                      long long* slot_stamp, unsigned char* routed, long long* step, int* miss,
                      int* n_miss, int policy, int decay, void* out_ids, int out_elem_bytes,
                      void* d0, const void* s0, long b0, void* d1, const void* s1, long b1,
                      void* d2, const void* s2, long b2, void* d3, const void* s3, long b3,
                      void* d4, const void* s4, long b4, void* d5, const void* s5, long b5,
                      int chunks, int lanes, int* sync, int max_wait_us, cudaStream_t stream) {
  if ((out_ids == nullptr && mk > 0) || (out_elem_bytes != 4 && out_elem_bytes != 8))
    return -1;
  if (sync == nullptr || (reinterpret_cast<uintptr_t>(sync) & 7) || max_wait_us < 0) return -1;
  if (S > EXPERT_CACHE_STEP_MAX_SLOTS) return -1;
  StepArgs a{};
  a.m = make_manage_args(topk_ids, mk, E, S, max_distinct, max_inserts, table, map_cold,
                         slot_expert, slot_stamp, routed, step, miss, n_miss, policy, decay);
  a.m.out_ids = mk > 0 ? out_ids : nullptr;
  a.m.out_elem_bytes = out_elem_bytes;
  if (!manage_args_ok(a.m)) return -1;
  void* dsts[EXPERT_CACHE_GATHER_SLOTS] = {d0, d1, d2, d3, d4, d5};
  const void* srcs[EXPERT_CACHE_GATHER_SLOTS] = {s0, s1, s2, s3, s4, s5};
  const long bytes[EXPERT_CACHE_GATHER_SLOTS] = {b0, b1, b2, b3, b4, b5};
  int rc = make_gather_args(dsts, srcs, bytes, miss, n_miss, &a.g);
  if (rc != 0) return rc;
  // the launch's tile counter is 32-bit: every tile index of the largest miss list fits
  if ((long long)a.g.tile_start[a.g.nbuf] * (max_inserts > 0 ? max_inserts : 1) >= INT_MAX)
    return -1;
  if (chunks <= 0 || lanes <= 0) return -1;
  a.chunks = chunks;
  a.lanes = lanes;
  a.sync = sync;
  a.wait_ns = 1000LL * (max_wait_us > 0 ? max_wait_us : EXPERT_CACHE_STEP_DEFAULT_WAIT_US);
  return launch_step(a, stream);
}

int expert_cache_manage_ep(const int* topk_ids, int mk, const int* expert_map, int E_global,
                           int E, int S, int max_distinct, int max_inserts, int* table,
                           int* map_cold, int* slot_expert, long long* slot_stamp,
                           unsigned char* routed, long long* step, int* miss, int* n_miss,
                           int policy, int decay, int* out_map, cudaStream_t stream) {
  if (expert_map == nullptr || out_map == nullptr || E_global <= 0) return -1;
  ManageArgs a = make_manage_args(topk_ids, mk, E, S, max_distinct, max_inserts, table,
                                  map_cold, slot_expert, slot_stamp, routed, step, miss,
                                  n_miss, policy, decay);
  a.emap = expert_map;
  a.Eg = E_global;
  a.out_map = out_map;
  return manage_checked(a, stream);
}

int expert_cache_prefetch(const int* pred_ids, int mk, int E, int S, int max_distinct,
                          int max_inserts, int* table, int* map_cold, int* slot_expert,
                          long long* slot_stamp, unsigned char* routed, long long* step,
                          int* miss, int* n_miss, int policy, cudaStream_t stream) {
  ManageArgs a = make_manage_args(pred_ids, mk, E, S, max_distinct, max_inserts, table,
                                  map_cold, slot_expert, slot_stamp, routed, step, miss,
                                  n_miss, policy, 0);
  a.prefetch = 1;
  return manage_checked(a, stream);
}

int expert_cache_pregate(const void* x, int T, int ldx, int H, const void* gate_w, int E,
                         int k, int* out_ids, cudaStream_t stream) {
  if (T < 0 || H <= 0 || H % 8 || H > EXPERT_CACHE_PREGATE_MAX_HIDDEN || ldx < H || ldx % 8)
    return -1;
  if (E <= 0 || E > EXPERT_CACHE_PREGATE_MAX_EXPERTS || k <= 0 || k > 32) return -1;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(gate_w)) & 15) return -1;
  if (T == 0) return 0;
  if (x == nullptr || gate_w == nullptr || out_ids == nullptr) return -1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)T);
  cfg.blockDim = dim3(kPregateThreads);
  cfg.dynamicSmemBytes = (size_t)H * 2 + (size_t)E * 4;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return (int)cudaLaunchKernelEx(&cfg, pregate_kernel,
                                 static_cast<const __nv_bfloat16*>(x), ldx, H,
                                 static_cast<const __nv_bfloat16*>(gate_w), E, k, out_ids);
}

int expert_cache_gather(void* d0, const void* s0, long b0, void* d1, const void* s1,
                        long b1, void* d2, const void* s2, long b2, void* d3,
                        const void* s3, long b3, void* d4, const void* s4, long b4,
                        void* d5, const void* s5, long b5, const int* miss,
                        const int* n_miss, int chunks, int lanes, cudaStream_t stream) {
  void* dsts[EXPERT_CACHE_GATHER_SLOTS] = {d0, d1, d2, d3, d4, d5};
  const void* srcs[EXPERT_CACHE_GATHER_SLOTS] = {s0, s1, s2, s3, s4, s5};
  const long bytes[EXPERT_CACHE_GATHER_SLOTS] = {b0, b1, b2, b3, b4, b5};
  GatherArgs a{};
  int rc = make_gather_args(dsts, srcs, bytes, miss, n_miss, &a);
  if (rc != 0) return rc;
  unsigned grid = 0;
  rc = gather_grid(chunks, lanes, &grid);
  if (rc != 0) return rc;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGatherThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return (int)cudaLaunchKernelEx(&cfg, gather_kernel, a);
}

}  // extern "C"
