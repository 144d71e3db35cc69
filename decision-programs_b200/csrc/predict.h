// Prediction with a trained ensemble over a dense fp32 device matrix: the
// kernels behind XGBoosterPredictFromCudaArray.
#pragma once
#include "kernels.h"

namespace dp {

// One tree node on the device.  Leaves have left < 0 and their value in cond.
struct PredNode {
  float cond;    // split threshold (x < cond goes left), or the leaf value
  i32 left;      // child ids within the tree; -1 at a leaf
  i32 right;
  u32 feat_dl;   // split feature | default_left << 31
};
static_assert(sizeof(PredNode) == 16, "prediction node layout");

// margin[r][k] = base[k] + the leaves of trees [t_begin, t_end) of class k,
// added in tree order (the order the training rounds added them).  Routing:
// x < cond goes left; a missing value (NaN, or mv when has_mv) follows
// default_left.  tree_off[t] is the first node of tree t, tree_off[t + 1] its
// end.  A walk longer than its tree sets bad[0] (a malformed model) and stops.
void launch_predict_margins(const float* x, u64 R, u64 stride, bool has_mv, float mv, const PredNode* nodes,
                            const u32* tree_off, const u32* tree_class, u32 t_begin, u32 t_end, int K,
                            const float* base, float* margin, u32* bad, cudaStream_t s);

// Objective transform of margins [R][K]: identity (squared error, width 1),
// sigmoid (logistic, width 1), softmax probabilities (softprob, width K),
// class index as float (softmax, width 1, first maximum on ties).  The
// arithmetic is the gradients' own: double, this library's exp, rounded to
// float.
void launch_predict_transform(int objective, int K, const float* margin, u64 R, float* out, cudaStream_t s);

}  // namespace dp
