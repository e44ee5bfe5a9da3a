// Top-1 MoE layer: not yet on the B200 path in this build.
#include "moe.h"

namespace nsb {

int moe_plan(ns_model*, Op&, int, bool) { return 0; }
int moe_forward(ns_model*, Op&, int, bool) { return -1; }
int moe_backward(ns_model*, Op&, int) { return -1; }
void moe_release(Op& op) { op.moe = nullptr; }

}  // namespace nsb
