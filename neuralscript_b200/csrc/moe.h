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


// Expert lifecycle on the device blob w (the reference CPU runtime's
// semantics, src/codegen/codegen.cpp:2559-2625). Geometry: gate [dim, cap]
// at off_g, experts e1 (and e2 unless linear) of n1 floats each.
struct ExpertGeom {
    size_t cap, dim, n1, off_g, off_e1, off_e2;
    bool linear;
};
// expert a := (a + b) / 2, gate column and expert matrices
int expert_merge_device(float* w, const ExpertGeom& g, int a, int b, cudaStream_t s);
// expert e := expert src + noise (noise: dim gate values, then n1 for e1,
// then n1 for e2 unless linear, in that order, already in device memory)
int expert_birth_device(float* w, const ExpertGeom& g, int src, int e, const float* noise, cudaStream_t s);

}  // namespace nsb
