// Host-side evaluation of the schedule chooser's boosted trees (the node
// arrays of ragged/selection.py TreeChooser): one walk per tree in C, so a
// call whose shape the runtime has not seen before pays a few microseconds
// for its choice instead of a NumPy walk of every tree.
#include <cstdint>

#include "internal.h"

using namespace rgb;

extern "C" int rg_tree_scores(int64_t nodes, const int32_t *feature, const double *threshold, const int32_t *left,
                              const int32_t *right, const double *value, const uint8_t *leaf, int64_t trees,
                              const int32_t *roots, const int32_t *tree_class, int classes,
                              const double *baseline, int features, const double *x, int max_depth,
                              double *scores) {
  if (nodes <= 0 || trees <= 0 || classes <= 0 || features <= 0 || max_depth < 0 || !feature || !threshold ||
      !left || !right || !value || !leaf || !roots || !tree_class || !baseline || !x || !scores)
    return fail(RG_ERR_INVALID_ARGUMENT, "rg_tree_scores: missing array or empty model");
  // Leaf values are summed per class in tree order from zero and the
  // baseline added last (the order of the NumPy walk, so both round alike).
  for (int c = 0; c < classes; ++c) scores[c] = 0.0;
  for (int64_t t = 0; t < trees; ++t) {
    int64_t node = roots[t];
    const int32_t cls = tree_class[t];
    if (cls < 0 || cls >= classes) return fail(RG_ERR_INVALID_ARGUMENT, "rg_tree_scores: tree class out of range");
    for (int depth = 0;; ++depth) {
      if (node < 0 || node >= nodes) return fail(RG_ERR_INVALID_ARGUMENT, "rg_tree_scores: node out of range");
      if (leaf[node]) break;
      if (depth == max_depth) return fail(RG_ERR_INVALID_ARGUMENT, "rg_tree_scores: tree deeper than max_depth");
      const int32_t f = feature[node];
      if (f < 0 || f >= features) return fail(RG_ERR_INVALID_ARGUMENT, "rg_tree_scores: feature out of range");
      node = x[f] <= threshold[node] ? left[node] : right[node];
    }
    scores[cls] += value[node];
  }
  for (int c = 0; c < classes; ++c) scores[c] = baseline[c] + scores[c];
  return RG_OK;
}
