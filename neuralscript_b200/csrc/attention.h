// Attention core launchers (see attention.cu for the layout contract).
#pragma once
#include <cuda_runtime.h>

namespace nsb {

struct AttnArgs {
    int B = 0, S = 0, H = 0, D = 0, dh = 0;
    float scale = 1.f;
    int dtype = 0;  // kF32 or kBF16 for qkv/ctx/dctx/dqkv
    const void* qkv = nullptr;
    long long ld_qkv = 0;
    void* ctx = nullptr;  // forward output; backward input (O)
    long long ld_ctx = 0;
    float* lse = nullptr;   // [B*H*S] log-sum-exp of each score row
    const void* dctx = nullptr;
    long long ld_dctx = 0;
    void* dqkv = nullptr;   // [M, ld] dQ | dK | dV
    long long ld_dqkv = 0;
    float* dvec = nullptr;  // [B*H*S] scratch: dO_i . O_i
    int* err = nullptr;     // device error word for bounded waits (tensor-core path)
};

int attention_fwd(const AttnArgs& a, cudaStream_t s);
// tcgen05 forward (attention_tc.cu): bf16, head dim 64, S <= 256
bool attention_tc_supported(const AttnArgs& a);
int attention_tc_fwd(const AttnArgs& a, cudaStream_t s, int* err);
// tcgen05 backward: bf16, head dim 64, S <= 256, lse from the forward
bool attention_tc_bwd_supported(const AttnArgs& a);
int attention_tc_bwd(const AttnArgs& a, cudaStream_t s, int* err);
// Number of kernel launches attention_bwd issues for `a`.
int attention_bwd_launches(const AttnArgs& a);
int attention_bwd(const AttnArgs& a, cudaStream_t s);

}  // namespace nsb
