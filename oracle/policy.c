/* Plain-C restatement of one expert-cache manage step.  TEST INFRASTRUCTURE ONLY.
 *
 * Same rules and the same state layout as oracle/policy.py (whose docstring cites the
 * reference line for each rule: kernels/expert_cache.hip:191-282 and 106-189,
 * tests/test_policy.py:83-132, vllm_expert_cache/cache.py:108-110).  This file exists
 * because the 4096-step traces and the timed CPU baseline want a compiled checker; it is
 * validated against the golden fixtures exactly like the Python one.
 *
 * Build: oracle/build.py (gcc -O2 -shared -fPIC) -> oracle/_build/liboracle.so
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OR_MAX_SLOTS 1024
#define OR_MAX_INSERTS 1024
#define OR_SLOT_BITS 20

typedef struct {
  int64_t stamp;
  int32_t slot;
} victim_key;

static int cmp_key(const void* a, const void* b) {
  const victim_key* x = (const victim_key*)a;
  const victim_key* y = (const victim_key*)b;
  if (x->stamp != y->stamp) return x->stamp < y->stamp ? -1 : 1;
  return (x->slot > y->slot) - (x->slot < y->slot);
}

/* Returns 0 on success, -1 when the launcher would refuse the arguments
 * (expert_cache.hip:596-598). `scratch_missing` must hold E ints. */
int oracle_manage(const int32_t* ids, int mk, int E, int S, int max_distinct,
                  int max_inserts, int32_t* table, int32_t* map_cold,
                  int32_t* slot_expert, int64_t* slot_stamp, uint8_t* routed,
                  int64_t* step, int32_t* miss, int32_t* n_miss, int policy, int decay) {
  if (E <= 0 || S <= 0 || S > OR_MAX_SLOTS || S > (1 << OR_SLOT_BITS) - 1) return -1;
  if (max_inserts < 0 || max_inserts > OR_MAX_INSERTS) return -1;
  if (policy < 0 || policy > 1) return -1;

  step[0] += 1;
  const int64_t now = step[0];
  n_miss[0] = 0;

  memset(routed, 0, (size_t)E);
  for (int i = 0; i < mk; i++) {
    const int e = ids[i];
    if (e >= 0 && e < E) routed[e] = 1;
  }
  int distinct = 0;
  for (int e = 0; e < E; e++) distinct += routed[e];
  if (distinct > max_distinct) return 0;

  int* missing = (int*)malloc(sizeof(int) * (size_t)(distinct > 0 ? distinct : 1));
  int nmissing = 0;
  for (int e = 0; e < E; e++) {
    if (!routed[e]) continue;
    const int s = table[e];
    if (s >= 0)
      slot_stamp[s] = (policy == 0) ? now : slot_stamp[s] + 1;
    else
      missing[nmissing++] = e;
  }
  const int nins = nmissing < max_inserts ? nmissing : max_inserts;
  if (nins <= 0) {
    free(missing);
    return 0;
  }
  for (int j = 0; j < nins; j++) miss[2 * j] = missing[j];

  if (policy != 0 && decay > 0 && (now % (int64_t)decay) == 0)
    for (int i = 0; i < S; i++) slot_stamp[i] >>= 1;

  victim_key* keys = (victim_key*)malloc(sizeof(victim_key) * (size_t)S);
  int nev = 0;
  for (int i = 0; i < S; i++) {
    const int x = slot_expert[i];
    if (x >= 0 && x < E && routed[x]) continue;
    keys[nev].stamp = slot_stamp[i];
    keys[nev].slot = i;
    nev++;
  }
  qsort(keys, (size_t)nev, sizeof(victim_key), cmp_key);
  const int nact = nins < nev ? nins : nev;
  const int64_t fresh = (policy == 0) ? now : 1;
  for (int r = 0; r < nact; r++) {
    const int sl = keys[r].slot;
    const int e = missing[r];
    const int old = slot_expert[sl];
    if (old >= 0) {
      table[old] = -1;
      map_cold[old] = old;
    }
    slot_expert[sl] = e;
    slot_stamp[sl] = fresh;
    table[e] = sl;
    map_cold[e] = -1;
    miss[2 * r + 1] = sl;
  }
  n_miss[0] = nact;
  free(keys);
  free(missing);
  return 0;
}

/* table[ids] with torch's negative wrap; -1 for ids outside [-E, E). */
void oracle_remap(const int32_t* ids, int mk, int E, const int32_t* table, void* out,
                  int out_elem_bytes) {
  for (int i = 0; i < mk; i++) {
    int64_t e = ids[i];
    int64_t v = -1;
    if (e >= -(int64_t)E && e < (int64_t)E) v = table[e < 0 ? e + E : e];
    if (out_elem_bytes == 8)
      ((int64_t*)out)[i] = v;
    else
      ((int32_t*)out)[i] = (int32_t)v;
  }
}

/* Replays `nsteps` calls; step t reads ids[t*mk .. t*mk+mk).  Records n_miss per step
 * in `nmiss_out` and returns the total number of installs (or -1 on refused args). */
long long oracle_run(const int32_t* ids, int nsteps, int mk, int E, int S,
                     int max_distinct, int max_inserts, int32_t* table, int32_t* map_cold,
                     int32_t* slot_expert, int64_t* slot_stamp, uint8_t* routed,
                     int64_t* step, int32_t* miss, int32_t* n_miss, int policy, int decay,
                     int32_t* nmiss_out) {
  long long total = 0;
  for (int t = 0; t < nsteps; t++) {
    if (oracle_manage(ids + (size_t)t * mk, mk, E, S, max_distinct, max_inserts, table,
                      map_cold, slot_expert, slot_stamp, routed, step, miss, n_miss,
                      policy, decay))
      return -1;
    if (nmiss_out) nmiss_out[t] = n_miss[0];
    total += n_miss[0];
  }
  return total;
}

/* CPU equivalent of one gather: dst_k[slot] = src_k[expert] for every installed miss. */
void oracle_gather(int nbuf, void* const* dsts, const void* const* srcs,
                   const long* nbytes, const int32_t* miss, const int32_t* n_miss) {
  for (int j = 0; j < n_miss[0]; j++) {
    const long e = miss[2 * j], sl = miss[2 * j + 1];
    for (int k = 0; k < nbuf; k++)
      memcpy((char*)dsts[k] + sl * nbytes[k], (const char*)srcs[k] + e * nbytes[k],
             (size_t)nbytes[k]);
  }
}
