/*
 * actune_router -- per-request precision routing on the host (C ABI, part of
 * libactune_b200.so; no GPU needed).
 *
 * Replaces the reference's Python routing of each request:
 *   PrecisionTree.route / route_vector   actune/tree.py:102-141
 *   action_forecast_features             actune/features.py:46-96
 * The selector tree is a binary tree of depth <= 5 over x = [13 action-history
 * features of the previous chunk, proprioceptive state], x[feature] <= threshold
 * going left, each node carrying a configuration index into
 * CONFIGURATIONS = (q00, q01, q11, q10) (tree.py:13).  A request without history,
 * with a state of the wrong length or with any non-finite input routes to the
 * tree's fallback configuration (tree.py:120-141).
 */
#ifndef ACTUNE_ROUTER_H
#define ACTUNE_ROUTER_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ACTUNE_ROUTER_OK 0
#define ACTUNE_ROUTER_INVALID 1      /* malformed tree, argument or non-finite action chunk */
#define ACTUNE_ACTION_FEATURES 13
#define ACTUNE_MAX_STATE_DIM 64

typedef struct actune_tree actune_tree;

/* Builds a tree from parallel node arrays (node 0 is the root): feature[i] < 0
 * marks a leaf, else left[i] / right[i] are child indices; profile_index[i] in
 * 0..3 for every node; fallback in 0..3.  Validated like PrecisionTree.__init__
 * (tree.py:105-118): depth <= 5, split features in [0, 13 + state_dim), finite
 * thresholds, both children present, every node reached once. */
int actune_tree_create(const int32_t* feature, const double* threshold, const int32_t* left, const int32_t* right,
                       const int32_t* profile_index, int32_t n_nodes, int32_t state_dim, int32_t fallback,
                       actune_tree** out);
void actune_tree_destroy(actune_tree* tree);

/* Routes `batch` requests: features [batch, 13] (NULL: no history for any),
 * has_history [batch] (NULL: all have history), states [batch, state_len].
 * Writes each request's configuration index and reached leaf node (-1 for the
 * fallback); leaf may be NULL. */
int actune_tree_route_batch(const actune_tree* tree, const double* features, const uint8_t* has_history,
                            const double* states, int32_t state_len, int32_t batch, int32_t* configuration,
                            int32_t* leaf);

/* The 13 action features of one [horizon, 7] chunk (row-major doubles) and its
 * gripper margin, in the order of ACTION_FORECAST_FEATURE_NAMES
 * (features.py:4-18).  ACTUNE_ROUTER_INVALID for a non-finite input. */
int actune_action_features(const double* actions, int32_t horizon, double gripper_margin, double* out);

#ifdef __cplusplus
}
#endif

#endif /* ACTUNE_ROUTER_H */
