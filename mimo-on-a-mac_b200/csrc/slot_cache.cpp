// Expert residency table: which experts of a layer sit in its S device slots, and which slots to refill
// when a step needs experts that are not resident (engine/mimo_stream/cache.py:13-65, SlotCache).
//
// Policy (the reference's decayed LFU): every resolve is one tick; each needed expert's count rises by one
// (when counted) and its last-use tick is set; the missing experts take the slots with the lowest score
// count * 1e12 + last-use tick (an empty slot scores -1, a slot holding a needed expert is never taken);
// decay() halves every count (the engine calls it every 16 decode tokens, model.py:348-354).  The reference
// picks victims with np.argpartition, which leaves their order and the choice among equal scores open; here
// victims are taken in ascending (score, slot) order and the i-th missing expert (in the order given) goes
// to the i-th victim.
//
// Differences from the reference, both on inputs it does not check: a step needing more distinct experts
// than there are slots returns MIMO_ERANGE before changing anything (the reference raises only when the
// missing experts alone exceed the slots, and can otherwise evict one of the step's own experts), and
// repeated or out-of-range expert ids return MIMO_EINVAL.  preload() keeps the table consistent when called
// on a table that already holds experts (each moved expert and each overwritten slot is unmapped first).
//
// Host code only: the copies into the slots and the kernels' slot indirection are the caller's
// (mimo_moe.residency.ExpertCache).  One table per layer; not thread-safe.
#include <algorithm>
#include <cstdint>
#include <limits>
#include <new>
#include <vector>

#include "../../include/mimo_moe.h"

namespace {

struct SlotTable {
  int32_t S, E;
  std::vector<int32_t> slot_of;    // expert -> slot or -1
  std::vector<int32_t> expert_in;  // slot -> expert or -1
  std::vector<double> cnt;         // decayed selection count per expert
  std::vector<int64_t> last;       // tick of the last resolve that needed the expert
  int64_t t = 0, hits = 0, misses = 0;
  std::vector<uint8_t> mark;       // scratch: ids seen in the current call
  std::vector<int32_t> missing, order;
  std::vector<double> score;

  SlotTable(int32_t s, int32_t e)
      : S(s), E(e), slot_of(e, -1), expert_in(s, -1), cnt(e, 0.0), last(e, 0), mark(e, 0), score(s) {}

  // ids in [0, E) and pairwise distinct
  bool distinct_ids(const int32_t* ids, int32_t n) {
    bool ok = true;
    int32_t i = 0;
    for (; i < n; ++i) {
      const int32_t e = ids[i];
      if (e < 0 || e >= E || mark[e]) {
        ok = false;
        break;
      }
      mark[e] = 1;
    }
    for (int32_t j = 0; j < i; ++j) mark[ids[j]] = 0;
    return ok;
  }

  void assign(int32_t e, int32_t s) {
    const int32_t old = expert_in[s];
    if (old >= 0) slot_of[old] = -1;
    if (slot_of[e] >= 0) expert_in[slot_of[e]] = -1;
    expert_in[s] = e;
    slot_of[e] = s;
  }
};

SlotTable* table(void* h) { return static_cast<SlotTable*>(h); }

}  // namespace

extern "C" {

void* mimo_moe_slot_cache_create(int32_t n_slots, int32_t n_experts) {
  if (n_slots < 1 || n_experts < 1 || n_slots > n_experts || n_experts > (1 << 20)) return nullptr;
  return new (std::nothrow) SlotTable(n_slots, n_experts);
}

void mimo_moe_slot_cache_destroy(void* h) { delete table(h); }

int mimo_moe_slot_cache_preload(void* h, const int32_t* experts, int32_t n, int32_t* load_expert,
                                int32_t* load_slot, int32_t* n_loads) {
  SlotTable* c = table(h);
  if (!c || n < 0 || (n > 0 && !experts) || !n_loads) return MIMO_EINVAL;
  const int32_t m = std::min(n, c->S);
  if ((m > 0 && (!load_expert || !load_slot)) || !c->distinct_ids(experts, m)) return MIMO_EINVAL;
  for (int32_t s = 0; s < m; ++s) {
    c->assign(experts[s], s);
    load_expert[s] = experts[s];
    load_slot[s] = s;
  }
  *n_loads = m;
  return MIMO_OK;
}

int mimo_moe_slot_cache_resolve(void* h, const int32_t* needed, int32_t n, int32_t count, int32_t stats,
                                int32_t* load_expert, int32_t* load_slot, int32_t* n_loads) {
  SlotTable* c = table(h);
  if (!c || n < 0 || (n > 0 && (!needed || !load_expert || !load_slot)) || !n_loads) return MIMO_EINVAL;
  if (!c->distinct_ids(needed, n)) return MIMO_EINVAL;
  if (n > c->S) return MIMO_ERANGE;
  *n_loads = 0;
  c->t += 1;
  c->missing.clear();
  for (int32_t i = 0; i < n; ++i) {
    const int32_t e = needed[i];
    if (count) c->cnt[e] += 1.0;
    c->last[e] = c->t;
    if (c->slot_of[e] < 0) c->missing.push_back(e);
  }
  const int32_t m = static_cast<int32_t>(c->missing.size());
  if (stats) {
    c->hits += n - m;
    c->misses += m;
  }
  if (m == 0) return MIMO_OK;
  for (int32_t s = 0; s < c->S; ++s) {
    const int32_t e = c->expert_in[s];
    c->score[s] = e >= 0 ? c->cnt[e] * 1e12 + static_cast<double>(c->last[e]) : -1.0;
  }
  for (int32_t i = 0; i < n; ++i) {
    const int32_t s = c->slot_of[needed[i]];
    if (s >= 0) c->score[s] = std::numeric_limits<double>::infinity();
  }
  c->order.resize(c->S);
  for (int32_t s = 0; s < c->S; ++s) c->order[s] = s;
  const std::vector<double>& sc = c->score;
  std::partial_sort(c->order.begin(), c->order.begin() + m, c->order.end(), [&sc](int32_t a, int32_t b) {
    return sc[a] < sc[b] || (sc[a] == sc[b] && a < b);
  });
  for (int32_t i = 0; i < m; ++i) {
    const int32_t e = c->missing[i], s = c->order[i];
    c->assign(e, s);
    load_expert[i] = e;
    load_slot[i] = s;
  }
  *n_loads = m;
  return MIMO_OK;
}

int mimo_moe_slot_cache_decay(void* h) {
  SlotTable* c = table(h);
  if (!c) return MIMO_EINVAL;
  for (double& v : c->cnt) v *= 0.5;
  return MIMO_OK;
}

int mimo_moe_slot_cache_state(void* h, int32_t* slot_of, int32_t* expert_in, int64_t* hits, int64_t* misses) {
  SlotTable* c = table(h);
  if (!c) return MIMO_EINVAL;
  if (slot_of) std::copy(c->slot_of.begin(), c->slot_of.end(), slot_of);
  if (expert_in) std::copy(c->expert_in.begin(), c->expert_in.end(), expert_in);
  if (hits) *hits = c->hits;
  if (misses) *misses = c->misses;
  return MIMO_OK;
}

}  // extern "C"
