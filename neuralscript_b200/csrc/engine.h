// Engine internals shared by engine.cpp and the MoE layer (moe.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <nccl.h>
#include <stdint.h>

#include <random>
#include <string>
#include <vector>

#include "spec.h"

struct ns_model;

namespace nsb {

// Kernel launches issued by the calling thread (each launcher adds its own).
long long& launch_counter();

enum OpKind {
    OP_DENSE, OP_EMB, OP_ATTN, OP_LN, OP_MOE, OP_ADD, OP_SUB, OP_MUL, OP_DIV, OP_ACT, OP_SOFTMAX, OP_DROPOUT,
    OP_CONCAT, OP_SLICE, OP_INDEX, OP_SCATTER
};

struct Val {
    std::string name;
    int cols = 0;
    int producer = -1;  // op index, -1 for the input
    std::vector<int> consumers;
    bool need_f32 = true, need_h16 = false;
    bool materialized = true;  // false: a dense output folded into a residual add
    int alias_of = -1;         // dropout: storage shared with its input
    bool ln_hidden = false;    // a residual sum normalised inside its producer's GEMM: never stored
    float* f32 = nullptr;
    __nv_bfloat16* h16 = nullptr;
    // backward
    float* gbuf = nullptr;
    const float* gcur = nullptr;
};

struct MoeScratch;

// allocation helper bound to a model's plan (freed on re-plan / free)
void* plan_alloc(ns_model* m, size_t bytes);

// Per-region timing around part of an operation (no-op unless the model's
// region timing is on): the index from region_open goes to region_close.
int region_open(ns_model* m, const std::string& label);
void region_close(ns_model* m, int idx);

struct Op {
    int kind = OP_DENSE;
    int layer = -1;
    int act = 0;
    int in = -1, in2 = -1, out = -1;  // value indices (out = the value written)
    int self_out = -1;                // the op's own output value (differs from out when fused)
    bool skip = false;                // an add folded into its producer's epilogue
    int fused_res = -1;               // residual value added in the epilogue
    int widx = -1;                    // first weight index of the layer
    // dense / attention scratch
    void* z = nullptr;  // pre-activation (training)
    void* dz = nullptr;
    float* dz32 = nullptr;
    void* qkv = nullptr;
    void* ctx = nullptr;
    void* dqkv = nullptr;
    void* dctx = nullptr;
    void* dout_w = nullptr;
    float* lse = nullptr;
    float* dvec = nullptr;
    MoeScratch* moe = nullptr;
    // data movement: integer operands (slice bounds / column indices), the
    // indices also on the device (int64, as the reference's kernels take them)
    std::vector<long long> ints;
    int64_t* d_idx = nullptr;
    float drop_rate = 0.f;  // dropout layers
    int drop_site = 0;      // dropout: index among the network's dropout ops
    // LayerNorm fused into this op's GEMM (the op's output r = residual sum
    // feeds only a LayerNorm, N = 512): ln_op is that LayerNorm's index, the
    // GEMM writes its output and ln_rstd; on the LayerNorm, ln_from is the
    // producer's index (forward skipped, backward from the output)
    int ln_op = -1, ln_from = -1;
    float* ln_rstd = nullptr;
    bool dz_ready = false;  // backward: dz already holds act'(z) * dout (written by the consumer's GEMM)
    bool g16_ready = false;  // backward: dz / dout_w already holds the bf16 output gradient
};

}  // namespace nsb

namespace nsb {
struct ReplicaPool;
}

struct ns_model {
    nsb::Spec spec;
    // In-call multi-GPU (NS_B200_GPUS=N at init): the model on the first
    // device holds replicas on the others, joined by NCCL, and one worker
    // thread per replica; every ABI call splits its rows over all of them.
    std::vector<ns_model*> reps;
    nsb::ReplicaPool* pool = nullptr;
    int device = 0;
    cudaStream_t stream = nullptr;
    int* d_err = nullptr;
    int precision = 2;
    int wdt = 1;  // working dtype of GEMM operands (kF32 / kBF16)
    // parameters
    float* d_w = nullptr;    // fp32 master blob
    float* d_g = nullptr;    // gradient blob (+1 trailing float: loss sum for the all-reduce)
    float* d_m = nullptr;    // AdamW first moment / Muon momentum
    float* d_v = nullptr;    // AdamW second moment
    float* d_o = nullptr;    // orthogonalisation scratch (largest matrix x 2)
    float* d_ns = nullptr;   // Newton-Schulz scratch
    size_t ns_floats = 0;
    std::vector<void*> wk;   // working copy per weight index (nullptr when unused)
    std::vector<bool> wk_owned;
    std::vector<long long> adam_t;
    // host mirror of the master blob
    mutable std::vector<float> h_w;
    mutable bool host_dirty = false;
    // MoE liveness
    int moe_layer = -1;
    std::vector<uint8_t> moe_active;
    size_t moe_active_count = 0;
    uint8_t* d_active = nullptr;
    std::mt19937 rng{0x9E3779B9u};
    long long lr_step = 0;
    uint32_t drop_key0 = 0x243F6A88u, drop_key1 = 0x85A308D3u;  // dropout Philox key
    uint32_t drop_step = 0;  // advances every training step (fresh masks per step)
    int last_rows = 0;       // rows of the last train step (input gradient export)
    bool seed16 = false;  // last loss seed went to the output Dense layer's bf16 dz
    bool ln_fusion = false;  // LayerNorms fused into their producers' GEMMs (tensor-core modes)
    // head GEMM + cross-entropy fusion (bf16 training with int32 targets):
    // the output layer's GEMM leaves bf16 logits in its dz buffer and the
    // fp32 target logits here; the loss pass turns the logits into the seed
    bool ce_fused = false;
    const int* ce_targets = nullptr;
    float* d_tlogit = nullptr;
    // graph
    std::vector<nsb::Val> vals;
    std::vector<nsb::Op> ops;
    int out_val = -1;
    // plan (sized for mmax rows)
    int mmax = 0;
    bool train_planned = false;
    std::vector<void*> plan_allocs;
    float* d_in = nullptr;
    float* d_labels = nullptr;
    int* d_targets = nullptr;
    int* h_targets = nullptr;  // pinned: one-hot label rows read back as class indices
    int h_targets_cap = 0;
    float* d_rowloss = nullptr;
    float* d_loss = nullptr;
    float* h_loss = nullptr;  // pinned
    float* d_ws = nullptr;    // split-K workspace
    size_t ws_floats = 0;
    // weight-gradient GEMMs of the backward on a second stream (bf16, one
    // rank): they overlap the input-gradient chain and join before the
    // optimizer; their split-K workspace is their own
    cudaStream_t wstream = nullptr;
    cudaEvent_t ev_ms = nullptr, ev_sm = nullptr;  // main -> side, side -> main
    float* d_ws2 = nullptr;
    size_t ws2_floats = 0;
    bool side_w = false;       // this backward uses the side stream
    bool side_used = false;    // ... and has launched on it
    cudaEvent_t ev_emb = nullptr;  // the embedding gradient's sort, done on the side stream
    int emb_sorted = -1;           // op whose sort ran ahead on the side stream (-1: none)
    void* d_scratch = nullptr;  // embedding-gradient sort scratch
    size_t scratch_bytes = 0;
    // data parallel
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
    bool group_lost = false;  // the communicator was aborted; train steps fail from then on
    cudaEvent_t ev_in = nullptr, ev_out = nullptr;  // ordering with the caller's stream (device entries)
    cudaStream_t comm_stream = nullptr;    // gradient all-reduces, overlapped with the backward
    // pipelined host-buffer inference: output rows staged per chunk and
    // copied to the caller on copy_stream while the next chunk computes
    cudaStream_t copy_stream = nullptr;
    float* d_stage = nullptr;  // plan allocation, mmax x out_cols
    std::vector<cudaEvent_t> chunk_events;
    std::vector<cudaEvent_t> dist_events;  // ordering events between the two streams
    size_t ev_next = 0;
    std::vector<char> reduced;             // per weight: its all-reduce was issued this step
    std::vector<std::pair<int, int>> bucket_w;  // weight ranges in all-reduce issue order
    std::vector<cudaEvent_t> bucket_done;       // recorded on the comm stream after each collective
    std::vector<cudaEvent_t> bucket_evt;        // per bucket (bucket_w): its last collective's event
    std::vector<int> owner;  // per weight: rank that updates it (sharded Muon) or -1 (replicated update)
    int timeout_ms = 60000;
    long long launches = 0;
    // per-region CUDA-event timing on the engine stream (opt-in)
    bool timing = false;
    struct Region {
        std::string label;
        std::vector<std::pair<cudaEvent_t, cudaEvent_t>> pending;
        std::vector<std::pair<cudaEvent_t, cudaEvent_t>> pool;
        double ms = 0;
        long long count = 0;
    };
    std::vector<Region> regions;
};
