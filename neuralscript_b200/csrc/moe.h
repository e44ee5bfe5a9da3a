// Top-1 mixture-of-experts layer on the engine (router, dispatch, grouped
// expert GEMMs, combine; backward).
#pragma once
#include "engine.h"

namespace nsb {

int moe_plan(ns_model* m, Op& op, int mmax, bool train);
int moe_forward(ns_model* m, Op& op, int M, bool train);
int moe_backward(ns_model* m, Op& op, int M);
void moe_release(Op& op);
int moe_route(const float* x, const float* Wg, const uint8_t* active, int M, int D, int E, int* best, float* pb,
              float* probs, cudaStream_t s);

}  // namespace nsb
