// K4 — expert-placement plan (host, integer, deterministic: every rank computes the same plan
// from the same all-gathered counts) and the send / receive layout derived from it.
#include <stdint.h>

#include <vector>

#include "../../include/dsca_b200.h"

namespace {

int argmax_first(const std::vector<int64_t>& v) {
  int b = 0;
  for (int i = 1; i < (int)v.size(); ++i)
    if (v[i] > v[b]) b = i;
  return b;
}
int argmin_first(const std::vector<int64_t>& v) {
  int b = 0;
  for (int i = 1; i < (int)v.size(); ++i)
    if (v[i] < v[b]) b = i;
  return b;
}

}  // namespace

// Scheduler.schedule_fixed + schedule_harmony (src/harmonymoe/scheduler.py:268-279, 324-372):
//   start from S[src, e, owner(e)] = meta[src, e]; avg = sum(meta) // G; while some GPU holds
//   more than avg: take the most loaded (first on ties) and the least loaded GPU; stop if they
//   coincide or the least loaded one cannot take eq_tokens more; take the expert with most
//   tokens on the overloaded GPU (stop if below eq_tokens); move tokens of that expert from its
//   largest senders first, each move bounded by the room left on the least loaded GPU, until the
//   overload is gone or the room is used up.
extern "C" int dsca_plan_harmony(const int32_t* meta, int G, int E, const int32_t* expert_to_gpu,
                                 int eq_tokens, int32_t* S) {
  if (meta == nullptr || expert_to_gpu == nullptr || S == nullptr || G <= 0 || E <= 0 ||
      G > DSCA_MAX_GPUS)
    return DSCA_ERR_BAD_ARG;
  std::vector<int64_t> s((size_t)G * E * G, 0);
  auto at = [&](int src, int e, int dst) -> int64_t& { return s[((size_t)src * E + e) * G + dst]; };
  int64_t total = 0;
  for (int src = 0; src < G; ++src)
    for (int e = 0; e < E; ++e) {
      int owner = expert_to_gpu[e];
      if (owner < 0 || owner >= G || meta[(size_t)src * E + e] < 0) return DSCA_ERR_BAD_ARG;
      at(src, e, owner) = meta[(size_t)src * E + e];
      total += meta[(size_t)src * E + e];
    }
  if (eq_tokens >= 0) {
    const int64_t avg = total / G;
    std::vector<int64_t> amt(G, 0);
    for (int src = 0; src < G; ++src)
      for (int e = 0; e < E; ++e)
        for (int dst = 0; dst < G; ++dst) amt[dst] += at(src, e, dst);
    for (;;) {
      bool over_any = false;
      for (int g = 0; g < G; ++g) over_any |= amt[g] > avg;
      if (!over_any) break;
      const int over = argmax_first(amt);
      const int least = argmin_first(amt);
      if (least == over || amt[least] + eq_tokens > avg) break;
      std::vector<int64_t> send(E, 0);
      for (int src = 0; src < G; ++src)
        for (int e = 0; e < E; ++e) send[e] += at(src, e, over);
      const int e = argmax_first(send);
      if (send[e] < eq_tokens) break;
      int64_t amount_over = amt[over] - avg;
      int64_t moved = 0;
      while (amount_over > 0 && avg - amt[least] > 0) {
        std::vector<int64_t> senders(G);
        for (int src = 0; src < G; ++src) senders[src] = at(src, e, over);
        const int src = argmax_first(senders);
        const int64_t tok = senders[src];
        if (tok <= 0) break;
        const int64_t n = tok < (avg - amt[least]) ? tok : (avg - amt[least]);
        at(src, e, over) -= n;
        at(src, e, least) += n;
        amt[over] -= n;
        amt[least] += n;
        amount_over -= n;
        moved += n;
      }
      if (moved == 0) break;  // guard: the reference would loop forever here
    }
  }
  for (size_t i = 0; i < s.size(); ++i) S[i] = (int32_t)s[i];
  return DSCA_OK;
}

// Send side (rank r): rows for dst in order, inside dst experts ascending
// (Scheduler.distribute_tokens, src/harmonymoe/scheduler.py:101-124).
// Receive side: expert-major, chunks (src ascending) inside each expert
// (Scheduler.generate_expert_mask, :185-213, with a stable order).
extern "C" int dsca_plan_layout(const int32_t* S, int G, int E, int rank, int* num_groups,
                                int32_t* group_expert, int32_t* group_offsets, int32_t* recv_off,
                                int32_t* send_base, int32_t* cum_split, int32_t* send_splits,
                                int32_t* recv_splits) {
  if (S == nullptr || num_groups == nullptr || group_expert == nullptr || group_offsets == nullptr ||
      recv_off == nullptr || send_base == nullptr || cum_split == nullptr || send_splits == nullptr ||
      recv_splits == nullptr || G <= 0 || E <= 0 || rank < 0 || rank >= G)
    return DSCA_ERR_BAD_ARG;
  auto at = [&](int src, int e, int dst) -> int32_t { return S[((size_t)src * E + e) * G + dst]; };
  // sender
  int32_t row = 0;
  for (int dst = 0; dst < G; ++dst) {
    int32_t n0 = row;
    for (int e = 0; e < E; ++e) {
      send_base[(size_t)e * G + dst] = row;
      row += at(rank, e, dst);
    }
    send_splits[dst] = row - n0;
  }
  for (int e = 0; e < E; ++e) {
    int32_t c = 0;
    for (int dst = 0; dst < G; ++dst) {
      c += at(rank, e, dst);
      cum_split[(size_t)e * G + dst] = c;
    }
  }
  // receiver
  int ng = 0;
  int32_t r = 0;
  for (int src = 0; src < G; ++src) {
    int32_t c = 0;
    for (int e = 0; e < E; ++e) c += at(src, e, rank);
    recv_splits[src] = c;
  }
  for (int src = 0; src < G; ++src)
    for (int e = 0; e < E; ++e) recv_off[(size_t)src * E + e] = -1;
  group_offsets[0] = 0;
  for (int e = 0; e < E; ++e) {
    int32_t c = 0;
    for (int src = 0; src < G; ++src) c += at(src, e, rank);
    if (c == 0) continue;
    group_expert[ng] = e;
    for (int src = 0; src < G; ++src) {
      int32_t n = at(src, e, rank);
      if (n > 0) recv_off[(size_t)src * E + e] = r;
      r += n;
    }
    ++ng;
    group_offsets[ng] = r;
  }
  *num_groups = ng;
  return DSCA_OK;
}
