// Per-request precision router (host code; declared in include/actune_router.h).
//
// The reference routes each request in Python: PrecisionTree.route
// (actune/tree.py:102-141) walks a depth <= 5 binary tree over 13 action-history
// features followed by the proprioceptive state, with a fallback configuration
// whenever the history or the state is missing, non-finite or of the wrong
// length; the 13 features come from the previous action chunk
// (actune/features.py:46-96).  Here both run as plain C++ over flat arrays: the
// tree is stored as parallel node arrays (feature, threshold, children, leaf
// configuration), validated once, and routed in a few dozen nanoseconds per
// request, batched over environments.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <new>
#include <vector>

#include "actune_router.h"

struct actune_tree {
  std::vector<int32_t> feature, left, right, profile;
  std::vector<double> threshold;
  int32_t state_dim = 0;
  int32_t fallback = 2;
};

namespace {

constexpr int kFeatures = ACTUNE_ACTION_FEATURES;
constexpr int kMaxDepth = 5;

bool valid_node(const actune_tree& t, int32_t i, int depth, int32_t n, std::vector<uint8_t>& seen) {
  if (i < 0 || i >= n || seen[i] || depth > kMaxDepth) return false;
  seen[i] = 1;
  if (t.profile[i] < 0 || t.profile[i] > 3) return false;
  if (t.feature[i] < 0) return t.left[i] < 0 && t.right[i] < 0;  // leaf
  if (t.feature[i] >= kFeatures + t.state_dim || !std::isfinite(t.threshold[i])) return false;
  if (t.left[i] < 0 || t.right[i] < 0) return false;
  return valid_node(t, t.left[i], depth + 1, n, seen) && valid_node(t, t.right[i], depth + 1, n, seen);
}

// Leaf reached by x (13 + state_dim finite values), walking from node 0:
// x[feature] <= threshold goes left (tree.py:123-126).
int32_t walk(const actune_tree& t, const double* x) {
  int32_t i = 0;
  while (t.feature[i] >= 0) i = x[t.feature[i]] <= t.threshold[i] ? t.left[i] : t.right[i];
  return i;
}

// Sum of n doubles in the order numpy's add.reduce uses for a contiguous 1-D array
// (pairwise summation: below 8 terms a running sum, up to 128 terms eight strided
// partial sums combined as ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) plus the tail,
// above that the halves recursively), so the row-norm means match np.mean.
double pairwise_sum(const double* v, int n) {
  if (n < 8) {
    double r = 0.0;
    for (int i = 0; i < n; ++i) r += v[i];
    return r;
  }
  if (n <= 128) {
    double r[8];
    for (int j = 0; j < 8; ++j) r[j] = v[j];
    int i = 8;
    for (; i < n - (n % 8); i += 8)
      for (int j = 0; j < 8; ++j) r[j] += v[i + j];
    double res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
    for (; i < n; ++i) res += v[i];
    return res;
  }
  int n2 = n / 2;
  n2 -= n2 % 8;
  return pairwise_sum(v, n2) + pairwise_sum(v + n2, n - n2);
}

// Euclidean norm of `width` consecutive values (a running sum of squares).
double row_norm(const double* v, int width) {
  double s = 0.0;
  for (int c = 0; c < width; ++c) s += v[c] * v[c];
  return std::sqrt(s);
}

// Of the [H x width] slice starting at column c0 of an [H x 7] chunk: the mean row
// norm, the mean norm of the first and second row differences (second differences
// taken as differences of the first ones, as np.diff(n=2) does) and the
// cancellation 1 - |sum of rows| / sum of row norms clipped to [0, 1]
// (features.py:22-43).
struct Motion {
  double energy, variation, curvature, cancellation;
};

Motion motion(const double* a, int H, int c0, int width) {
  Motion m{0.0, 0.0, 0.0, 0.0};
  std::vector<double> norms(H), d1((size_t)(H > 1 ? H - 1 : 0) * width);
  double total[6] = {0, 0, 0, 0, 0, 0};
  for (int r = 0; r < H; ++r) {
    norms[r] = row_norm(a + r * 7 + c0, width);
    for (int c = 0; c < width; ++c) total[c] = r == 0 ? a[c0 + c] : total[c] + a[r * 7 + c0 + c];
  }
  const double mag = pairwise_sum(norms.data(), H);
  m.energy = mag / H;
  if (H > 1) {
    std::vector<double> n1(H - 1);
    for (int r = 0; r + 1 < H; ++r) {
      for (int c = 0; c < width; ++c) d1[r * width + c] = a[(r + 1) * 7 + c0 + c] - a[r * 7 + c0 + c];
      n1[r] = row_norm(&d1[r * width], width);
    }
    m.variation = pairwise_sum(n1.data(), H - 1) / (H - 1);
  }
  if (H > 2) {
    std::vector<double> n2(H - 2), d2(width);
    for (int r = 0; r + 2 < H; ++r) {
      for (int c = 0; c < width; ++c) d2[c] = d1[(r + 1) * width + c] - d1[r * width + c];
      n2[r] = row_norm(d2.data(), width);
    }
    m.curvature = pairwise_sum(n2.data(), H - 2) / (H - 2);
  }
  const double canc = mag <= 1e-12 ? 0.0 : 1.0 - row_norm(total, width) / mag;
  m.cancellation = canc < 0.0 ? 0.0 : (canc > 1.0 ? 1.0 : canc);
  return m;
}

double sign(double v) { return v > 0.0 ? 1.0 : (v < 0.0 ? -1.0 : 0.0); }

}  // namespace

extern "C" {

int actune_tree_create(const int32_t* feature, const double* threshold, const int32_t* left, const int32_t* right,
                       const int32_t* profile_index, int32_t n_nodes, int32_t state_dim, int32_t fallback,
                       actune_tree** out) {
  if (out == nullptr) return ACTUNE_ROUTER_INVALID;
  *out = nullptr;
  if (n_nodes < 1 || n_nodes > 63 || state_dim < 1 || state_dim > ACTUNE_MAX_STATE_DIM || fallback < 0 || fallback > 3 || feature == nullptr ||
      threshold == nullptr || left == nullptr || right == nullptr || profile_index == nullptr)
    return ACTUNE_ROUTER_INVALID;
  actune_tree* t = new (std::nothrow) actune_tree();
  if (t == nullptr) return ACTUNE_ROUTER_INVALID;
  t->feature.assign(feature, feature + n_nodes);
  t->threshold.assign(threshold, threshold + n_nodes);
  t->left.assign(left, left + n_nodes);
  t->right.assign(right, right + n_nodes);
  t->profile.assign(profile_index, profile_index + n_nodes);
  t->state_dim = state_dim;
  t->fallback = fallback;
  std::vector<uint8_t> seen(n_nodes, 0);
  if (!valid_node(*t, 0, 0, n_nodes, seen)) {
    delete t;
    return ACTUNE_ROUTER_INVALID;
  }
  *out = t;
  return ACTUNE_ROUTER_OK;
}

void actune_tree_destroy(actune_tree* tree) { delete tree; }

int actune_tree_route_batch(const actune_tree* tree, const double* features, const uint8_t* has_history,
                            const double* states, int32_t state_len, int32_t batch, int32_t* configuration,
                            int32_t* leaf) {
  if (tree == nullptr || batch < 0 || configuration == nullptr || (batch > 0 && states == nullptr))
    return ACTUNE_ROUTER_INVALID;
  const int32_t S = tree->state_dim;
  double x[kFeatures + ACTUNE_MAX_STATE_DIM];
  for (int32_t b = 0; b < batch; ++b) {
    configuration[b] = tree->fallback;
    if (leaf) leaf[b] = -1;
    // Missing history, a state of the wrong length or a non-finite value: fallback.
    if (features == nullptr || (has_history != nullptr && !has_history[b]) || state_len != S) continue;
    bool finite = true;
    for (int f = 0; f < kFeatures && finite; ++f) finite = std::isfinite(x[f] = features[b * kFeatures + f]);
    for (int s = 0; s < S && finite; ++s) finite = std::isfinite(x[kFeatures + s] = states[(int64_t)b * S + s]);
    if (!finite) continue;
    const int32_t node = walk(*tree, x);
    configuration[b] = tree->profile[node];
    if (leaf) leaf[b] = node;
  }
  return ACTUNE_ROUTER_OK;
}

int actune_action_features(const double* actions, int32_t horizon, double gripper_margin, double* out) {
  if (actions == nullptr || out == nullptr || horizon < 1) return ACTUNE_ROUTER_INVALID;
  for (int64_t i = 0; i < (int64_t)horizon * 7; ++i)
    if (!std::isfinite(actions[i])) return ACTUNE_ROUTER_INVALID;
  if (!std::isfinite(gripper_margin)) return ACTUNE_ROUTER_INVALID;
  const Motion tr = motion(actions, horizon, 0, 3);
  const Motion rot = motion(actions, horizon, 3, 3);
  const Motion all = motion(actions, horizon, 0, 6);
  double transition = 0.0;
  for (int r = 1; r < horizon; ++r)
    if (sign(actions[r * 7 + 6]) != sign(actions[(r - 1) * 7 + 6])) transition = 1.0;
  const double values[kFeatures] = {tr.energy,       rot.energy,       tr.variation,    rot.variation,
                                    tr.curvature,    rot.curvature,    tr.cancellation, rot.cancellation,
                                    all.variation,   all.curvature,    all.cancellation, transition,
                                    gripper_margin};
  std::memcpy(out, values, sizeof(values));
  return ACTUNE_ROUTER_OK;
}

}  // extern "C"
