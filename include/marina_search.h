/*
 * marina_search: a batched PUCT search driving the evaluator, for the nodes/s measurement.
 *
 * Follows the reference's search (src/search/mod.rs, src/search/tree.rs): each search gathers
 * a batch of leaves by repeated descents that hold virtual visits (so later descents go
 * elsewhere), sends the batch to a network in one call, expands the leaves with the returned
 * priors and backs up value = W - L, negated at every ply. PUCT score
 * q + cpuct * prior * sqrt(N_parent) / (1 + n), with unvisited children at the parent's mean
 * minus fpu_reduction * sqrt(explored prior mass) (src/search/tree.rs:290-320). Terminal
 * leaves (mate, stalemate, fifty-move rule, bare kings / single minor) are backed up without
 * a network slot.
 *
 * Differences from the reference, which the harness does not need for a throughput figure:
 * descents place one visit each (the reference splits a budget per walk,
 * src/search/tree.rs:276-400, with the same sequential-PUCT semantics), and there are no
 * proofs, tablebases or repetition draws.
 */
#ifndef MARINA_SEARCH_H
#define MARINA_SEARCH_H

#include <stdint.h>

#include "marina_chess.h"

#ifdef __cplusplus
extern "C" {
#endif

/* A network: evaluate n packed positions (66-byte boards, 224 legal slots, -1 padded) into
 * priors [n, 224] and wdl [n, 3]. Returns 0 on success. `mrn_evaluate` has this signature. */
typedef int (*mrs_eval_fn)(void* ctx, int n, const uint8_t* boards, const int32_t* legal, float* priors, float* wdl);

typedef struct mrs_params {
  float cpuct;                  /* 1.75 (src/options.rs:303-307) */
  float fpu_reduction;          /* 0.25 */
  int32_t batch;                /* leaves per search per network call */
  int32_t batch_ramp;           /* a batch asks for at most tree size / ramp leaves (min 8); 0 = off */
  int32_t collision_budget_pct; /* stop gathering once collisions exceed this % of the batch */
} mrs_params;

typedef struct mrs_summary {
  uint64_t nodes;         /* leaves evaluated + terminal visits (Summary::nodes) */
  uint64_t network_evals; /* positions sent to a network */
  uint64_t batches;       /* network calls */
  uint64_t collisions;    /* descents that reached a leaf already in flight */
  uint64_t max_depth;
  uint64_t tree_nodes;    /* nodes allocated in the tree */
  double seconds;
  int32_t best_action;    /* most visited root move, as an action index */
  int32_t error;          /* 0, or the network's error code */
} mrs_summary;

/* Search `n_roots` positions to `node_limit` nodes each. Every one of `n_evaluators` networks
 * (e.g. one per GPU) is driven by `workers_per_evaluator` threads; roots are dealt to the
 * threads round-robin and each thread evaluates the leaves of all its roots in one network
 * call per round. Fills per-root summaries and the total (seconds = wall time). Returns 0, or
 * the first network error code. */
MRC_API int mrs_search(const mrc_position* roots, int n_roots, uint64_t node_limit, const mrs_params* params,
                       mrs_eval_fn eval, void* const* contexts, int n_evaluators, int workers_per_evaluator,
                       mrs_summary* per_root, mrs_summary* total);

/* `mrs_search`, also returning each root's children: `root_actions` and `root_visits` (both
 * n_roots x 224, -1 / 0 past the root's children) receive per root the action index and the visit
 * count of every child, in the root's move order -- the distribution the reference's search picks
 * its move from (most visits), for comparing searches driven by different networks. */
MRC_API int mrs_search_visits(const mrc_position* roots, int n_roots, uint64_t node_limit, const mrs_params* params,
                              mrs_eval_fn eval, void* const* contexts, int n_evaluators, int workers_per_evaluator,
                              mrs_summary* per_root, mrs_summary* total, int32_t* root_actions,
                              uint32_t* root_visits);

#ifdef __cplusplus
}
#endif

#endif /* MARINA_SEARCH_H */
