// Per-contraction operand precision.
//
// The session picks a precision (bf16 throughput mode, TF32 or TF32x3 accuracy modes); this pass
// turns it into one precision per FusedConv / FusedGemm, because the rounding error of tensor-core
// operands accumulates along chains of contractions that nothing averages away:
//
//  * A contraction is on a "dense chain" when its result reaches a graph output through ops that
//    keep one value per position (no global pooling or other reduction in between). ResNet's
//    convolutions feed a global average pool, so their per-pixel operand rounding errors average
//    out over 49 positions before the logits; a detector's per-anchor outputs (RetinaNet) carry the
//    error of every conv on their path.
//  * chain(op) = contractions on the longest dense chain through op, counted from the last global
//    pool (or the graph input) to the output; depth_in(op) = its position on that chain (1 = first).
//
// Measured against the fp32 oracle on RetinaNet-R50-FPN at its configured 800x1024 input (one
// image; chains of 57 convs), normwise error of the class / box outputs:
//   bf16 operands everywhere                     2.6e-2 / 1.7e-2   (bf16 gate 1e-2: missed)
//   bf16 in the 53 backbone convs, TF32 after    1.5e-2 / 9.6e-3   (at 128x160; the backbone alone
//                                                                   misses the gate)
//   bf16 in the first 16 / 12 / 8 / 4 convs, TF32 after
//                                                9.96e-3 / 8.2e-3 / 7.1e-3 / 4.9e-3 (class)
//   TF32 operands everywhere                     2.8e-3 / 2.5e-3   (TF32 gate 2e-3: missed)
//   TF32 in the backbone, fp32 in FPN and heads  2.5e-3 / 2.0e-3   (missed: the backbone alone)
//   TF32 in the first 32 / 24 / 16 / 8 convs, fp32 after
//                                                2.1e-3 / 1.6e-3 / 1.1e-3 / 7.5e-4 (class)
// The error grows about evenly per conv along the chain, so a long chain keeps the cheap operand
// type only for its first few contractions:
//  * bf16 sessions: on a dense chain of more than kDenseChain contractions, the ones past the first
//    kBf16Keep use TF32 operands (4.9e-3 on RetinaNet, a 2x margin to the bf16 gate). The MLP-6 and
//    StackedLinear chains (6 and 8) and every ResNet conv (pooled) stay bf16.
//  * TF32 sessions: on such a chain the contractions past the first kTf32Keep run as TF32x3
//    (error-compensated, near fp32): 1.1e-3, a 1.8x margin to the TF32 gate.
//  * TF32x3 sessions: every contraction TF32x3.
#include <algorithm>
#include <vector>

#include "ir.h"

namespace sb {

namespace {

bool is_contraction(const Op& op) { return !op.dead && (op.type == "FusedConv" || op.type == "FusedGemm"); }

// Ops after which per-position error no longer reaches the output one-to-one.
bool is_pooling(const Op& op) {
  return op.type == "GlobalAveragePool" || op.type == "GlobalMaxPool" || op.type == "ReduceMean" ||
         op.type == "ReduceSum" || op.type == "ReduceMax";
}

}  // namespace

constexpr int kDenseChain = 16;
constexpr int kBf16Keep = 4;
constexpr int kTf32Keep = 16;

void assign_precision(LGraph& g, int session_precision) {
  const int P = std::clamp(session_precision, 0, 2);
  for (Op& op : g.ops)
    if (is_contraction(op)) op.prec = P;
  if (P == 2) return;
  const size_t nv = g.vals.size();
  // depth_in: contractions since the last pooling op along the longest path to each value (ops are
  // in topological order).
  std::vector<int> din(nv, 0);
  for (const Op& op : g.ops) {
    if (op.dead) continue;
    int d = 0;
    if (!is_pooling(op)) {
      for (int id : op.in)
        if (id >= 0) d = std::max(d, din[size_t(id)]);
      if (op.residual >= 0) d = std::max(d, din[size_t(op.residual)]);
      if (op.concat >= 0) d = std::max(d, din[size_t(op.concat)]);
      if (is_contraction(op)) ++d;
    }
    for (int id : op.out)
      if (id >= 0) din[size_t(id)] = d;
  }
  // depth_out: contractions on the longest dense path from each value to a graph output (values
  // that reach no output without pooling: -1).
  std::vector<int> dout(nv, -1);
  for (int id : g.outputs) dout[size_t(id)] = 0;
  for (size_t i = g.ops.size(); i-- > 0;) {
    const Op& op = g.ops[i];
    if (op.dead || is_pooling(op)) continue;
    int d = -1;
    for (int id : op.out)
      if (id >= 0) d = std::max(d, dout[size_t(id)]);
    if (d < 0) continue;
    if (is_contraction(op)) ++d;
    auto up = [&](int id) {
      if (id >= 0) dout[size_t(id)] = std::max(dout[size_t(id)], d);
    };
    for (int id : op.in) up(id);
    up(op.residual);
    up(op.concat);
  }
  for (Op& op : g.ops) {
    if (!is_contraction(op)) continue;
    const int di = din[size_t(op.out[0])];          // position of op on its chain (1-based)
    const int dn = dout[size_t(op.out[0])];         // contractions after op on its dense path
    if (dn < 0) continue;                           // pooled before any output
    const int chain = di + dn;
    if (chain <= kDenseChain) continue;
    if (P == 0 && di > kBf16Keep) op.prec = 1;
    if (P == 1 && di > kTf32Keep) op.prec = 2;
  }
}

}  // namespace sb
