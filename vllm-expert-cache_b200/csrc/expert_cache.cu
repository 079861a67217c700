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
//                  torch gather/cast kernels of the Python remap disappear.
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
};

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

// NT threads; requires S <= NT.  Thread t owns slot t; experts are processed in tiles of
// NT (thread t owns expert base + t), in ascending id.
template <int NT>
__global__ void __launch_bounds__(NT) manage_kernel(const __grid_constant__ ManageArgs a) {
  constexpr int NW = NT / 32;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int s_missing[EXPERT_CACHE_MAX_INSERTS];   // r-th missing expert, ascending
  __shared__ int w_routed[2][NW], w_missed[2][NW], w_evict[NW];

  const int E = a.E, S = a.S;
  const int spad = (S + 1) & ~1;
  long long* s_key = reinterpret_cast<long long*>(smem);
  long long* s_st = s_key + spad;
  int* s_tab = reinterpret_cast<int*>(s_st + spad);
  int* s_se = s_tab + E;
  unsigned char* s_flag = reinterpret_cast<unsigned char*>(s_se + S);

  const int t = threadIdx.x, lane = t & 31, w = t >> 5;

  grid_dependency_wait();     // topk_ids may come from the kernel just before us
  release_dependents();       // let the gather launch and park on its own wait

  // ---- one round of loads: ids, step, table, slot state --------------------------------
  const long long now = a.step[0] + 1;
  const int my_id = (t < a.mk) ? a.ids[t] : -1;
  for (int e = t; e < E; e += NT) {
    s_tab[e] = a.table[e];
    s_flag[e] = 0;
  }
  for (int s = t; s < S; s += NT) {
    s_se[s] = a.slot_expert[s];
    s_st[s] = a.slot_stamp[s];
  }
  __syncthreads();
  if (t == 0) a.step[0] = now;   // every thread has read the old value above

  // ---- routed flags (duplicates write the same 1) ---------------------------------------
  if (my_id >= 0 && my_id < E) s_flag[my_id] = 1;
  for (int i = t + NT; i < a.mk; i += NT) {
    const int e = a.ids[i];
    if (e >= 0 && e < E) s_flag[e] = 1;
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
    if (hit) stamp = (a.policy == 0) ? now : stamp + 1;
  }
  {
    const unsigned b = __ballot_sync(0xffffffffu, t < S && !parked);
    if (lane == 0) w_evict[w] = __popc(b);
  }

  // ---- expert side: distinct count and the ascending miss list --------------------------
  int distinct = 0, n_missing = 0;
  for (int base = 0, tile = 0; base < E; base += NT, ++tile) {
    const int e = base + t;
    const bool f = e < E && s_flag[e];
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

  for (int e = t; e < E; e += NT) a.routed[e] = s_flag[e];

  const bool read_through = distinct > a.max_distinct;
  const int nins = read_through ? 0 : min(n_missing, a.max_inserts);
  if (nins == 0) {
    // Nothing to install: a read-through step changes no priority; otherwise the hits
    // keep their refreshed priority and no ageing runs (it only runs on inserting steps).
    if (!read_through && hit) a.slot_stamp[t] = stamp;
    if (t == 0) a.n_miss[0] = 0;
    if (a.out_ids) remap_tail(a.ids, a.mk, E, a.out_ids, a.out_elem_bytes, s_tab, my_id, NT);
    return;
  }

  // ---- ageing, eviction keys, miss list -------------------------------------------------
  const bool age = a.policy != 0 && a.decay > 0 && (now % (long long)a.decay) == 0;
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
  if (a.out_ids) {
    __syncthreads();
    remap_tail(a.ids, a.mk, E, a.out_ids, a.out_elem_bytes, s_tab, my_id, NT);
  }
}

// ---------------------------------------------------------------------------------------
// gather

constexpr int kGatherThreads = 256;
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

__global__ void __launch_bounds__(kGatherThreads)
    gather_kernel(const __grid_constant__ GatherArgs a) {
  const int per_miss = a.tile_start[a.nbuf];
  grid_dependency_wait();   // the miss list is written by the manage launch before us
  const long long total = (long long)a.n_miss[0] * per_miss;
  for (long long u = blockIdx.x; u < total; u += gridDim.x) {
    const int j = (int)(u / per_miss);
    const int v = (int)(u - (long long)j * per_miss);
    int k = 0;
    while (v >= a.tile_start[k + 1]) ++k;
    const long long first = (long long)(v - a.tile_start[k]) * kTileVecs;
    const long long left = a.vecs[k] - first;
    const long long e = a.miss[2 * j], s = a.miss[2 * j + 1];
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

// ---------------------------------------------------------------------------------------
// host side

int current_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= kMaxDevices) return -1;
  return d;
}

// Opt each manage instantiation into the full shared-memory carve-out once per device.
template <int NT>
cudaError_t ensure_manage_smem(int dev) {
  static bool done[kMaxDevices] = {};
  if (done[dev]) return cudaSuccess;
  int optin = 0;
  cudaError_t err = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (err != cudaSuccess) return err;
  cudaFuncAttributes fa{};
  err = cudaFuncGetAttributes(&fa, manage_kernel<NT>);
  if (err != cudaSuccess) return err;
  err = cudaFuncSetAttribute(manage_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             optin - (int)fa.sharedSizeBytes);
  if (err == cudaSuccess) done[dev] = true;
  return err;
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

int manage_checked(const ManageArgs& a, cudaStream_t stream) {
  if (a.E <= 0 || a.E > EXPERT_CACHE_MAX_EXPERTS) return -1;
  if (a.S <= 0 || a.S > EXPERT_CACHE_MAX_SLOTS || a.S > (1 << kSlotBits) - 1) return -1;
  if (a.max_inserts < 0 || a.max_inserts > EXPERT_CACHE_MAX_INSERTS) return -1;
  if (a.policy < 0 || a.policy > 1) return -1;
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
  return a;
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

int expert_cache_gather(void* d0, const void* s0, long b0, void* d1, const void* s1,
                        long b1, void* d2, const void* s2, long b2, void* d3,
                        const void* s3, long b3, void* d4, const void* s4, long b4,
                        void* d5, const void* s5, long b5, const int* miss,
                        const int* n_miss, int chunks, int lanes, cudaStream_t stream) {
  void* dsts[EXPERT_CACHE_GATHER_SLOTS] = {d0, d1, d2, d3, d4, d5};
  const void* srcs[EXPERT_CACHE_GATHER_SLOTS] = {s0, s1, s2, s3, s4, s5};
  const long bytes[EXPERT_CACHE_GATHER_SLOTS] = {b0, b1, b2, b3, b4, b5};
  for (int i = 0; i < EXPERT_CACHE_GATHER_SLOTS; ++i) {
    if (bytes[i] <= 0 || bytes[i] % 16) return -1;
    if ((reinterpret_cast<uintptr_t>(dsts[i]) | reinterpret_cast<uintptr_t>(srcs[i])) & 15)
      return -1;
  }
  if (chunks <= 0 || lanes <= 0) return -1;

  GatherArgs a{};
  int n = 0;
  long long tiles = 0;
  a.tile_start[0] = 0;
  for (int i = 0; i < EXPERT_CACHE_GATHER_SLOTS; ++i) {
    bool repeat = false;   // the caller pads to six by repeating a triple: copy it once
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

  const long long budget = (long long)chunks * (long long)lanes;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(budget < (1 << 20) ? budget : (1 << 20)));
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
