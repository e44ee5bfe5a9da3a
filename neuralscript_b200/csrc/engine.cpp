// NeuralScript B200 engine: plans buffers for a spec'd network once per row
// count, runs its forward pass, reverse-mode backward and optimizer step on
// one CUDA stream, all-reduces gradients over NCCL when data-parallel, and
// implements every ns_runtime.h entry point on top (the nsb_* functions).
//
// Reference behaviour followed (file:line in MrModelOS/NeuralScript):
//   forward launcher + C-ABI driver     src/codegen/codegen.cpp:552-1126
//   train core (fwd, grads, OPT_STEP)   src/codegen/codegen.cpp:3249-3653
//   CPU twin of both (the oracle)       src/codegen/codegen.cpp:2262-2657, 2755-3157
//   optimizer constants / LR schedule   include/ns/optim/optim_params.hpp:20-62
// Deliberate differences: per-sequence attention (`seq`), gradient SUM for
// values consumed twice (residuals), per-weight AdamW step counters on the
// device path too, no weight copy-back per step (lazy host mirror), checked
// CUDA errors (-1 through the unchanged ABI).
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <math.h>
#include <nccl.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/ns_b200.h"
#include "attention.h"
#include "elementwise.h"
#include "engine.h"
#include "gemm.h"
#include "kernels.h"
#include "moe.h"

using nsb::Op;
using nsb::Val;

namespace nsb {

long long& launch_counter() {
    static thread_local long long n = 0;
    return n;
}

static thread_local std::string g_err;

static int fail(const std::string& msg) {
    g_err = msg;
    return -1;
}

// NCCL is resolved at run time, only when data parallelism is requested:
// linking it would pin whichever libnccl.so.2 loads first for the whole
// process (PyTorch needs its own bundled build). An already-loaded copy is
// preferred.
struct Nccl {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*Reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, int, ncclComm_t,
                           cudaStream_t) = nullptr;
    ncclResult_t (*Broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*CommInitAll)(ncclComm_t*, int, const int*) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    bool ok = false;
};

static const Nccl& nccl() {
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        n.GetUniqueId = (decltype(n.GetUniqueId))dlsym(h, "ncclGetUniqueId");
        n.CommInitRankConfig = (decltype(n.CommInitRankConfig))dlsym(h, "ncclCommInitRankConfig");
        n.CommGetAsyncError = (decltype(n.CommGetAsyncError))dlsym(h, "ncclCommGetAsyncError");
        n.CommAbort = (decltype(n.CommAbort))dlsym(h, "ncclCommAbort");
        n.CommDestroy = (decltype(n.CommDestroy))dlsym(h, "ncclCommDestroy");
        n.AllReduce = (decltype(n.AllReduce))dlsym(h, "ncclAllReduce");
        n.Reduce = (decltype(n.Reduce))dlsym(h, "ncclReduce");
        n.Broadcast = (decltype(n.Broadcast))dlsym(h, "ncclBroadcast");
        n.CommInitAll = (decltype(n.CommInitAll))dlsym(h, "ncclCommInitAll");
        n.GetErrorString = (decltype(n.GetErrorString))dlsym(h, "ncclGetErrorString");
        n.ok = n.GetUniqueId && n.CommInitRankConfig && n.CommGetAsyncError && n.CommAbort && n.CommDestroy &&
               n.AllReduce && n.Reduce && n.Broadcast && n.CommInitAll && n.GetErrorString;
    });
    return n;
}

void* plan_alloc(ns_model* m, size_t bytes) {
    void* p = nullptr;
    // 4 KB of slack past every buffer: TMA boxes may read up to one 128-byte
    // swizzle row past a tensor's logical end.
    if (cudaMalloc(&p, bytes + 4096) != cudaSuccess) return nullptr;
    m->plan_allocs.push_back(p);
    return p;
}

static void* persist_alloc(size_t bytes) {
    void* p = nullptr;
    if (cudaMalloc(&p, bytes + 4096) != cudaSuccess) return nullptr;
    cudaMemset(p, 0, bytes + 4096);
    return p;
}

}  // namespace nsb

using namespace nsb;

// ---------------------------------------------------------------------------
// graph construction
// ---------------------------------------------------------------------------
static int find_val(ns_model* m, const std::string& n) {
    for (size_t i = 0; i < m->vals.size(); i++)
        if (m->vals[i].name == n) return (int)i;
    return -1;
}

static bool build_graph(ns_model* m, std::string& err) {
    Spec& s = m->spec;
    m->vals.clear();
    m->ops.clear();
    Val x;
    x.name = "x";
    x.cols = s.in_cols;
    m->vals.push_back(x);
    for (auto& so : s.ops) {
        Op op;
        if (so.fn == "add") op.kind = OP_ADD;
        else if (so.fn == "sub") op.kind = OP_SUB;
        else if (so.fn == "mul") op.kind = OP_MUL;
        else if (so.fn == "div") op.kind = OP_DIV;
        else if (so.fn == "concat") op.kind = OP_CONCAT;
        else if (so.fn == "slice") op.kind = OP_SLICE;
        else if (so.fn == "index") op.kind = OP_INDEX;
        else if (so.fn == "scatter") op.kind = OP_SCATTER;
        else if (so.fn == "softmax") op.kind = OP_SOFTMAX;
        else if (act_code(so.fn) >= 0) {
            op.kind = OP_ACT;
            op.act = act_code(so.fn);
        } else {
            op.layer = s.layer_index(so.fn);
            const LayerSpec& l = s.layers[op.layer];
            if (l.kind == "dense") {
                op.kind = OP_DENSE;
                op.act = act_code(l.gets("act", "identity"));
            } else if (l.kind == "embedding") op.kind = OP_EMB;
            else if (l.kind == "attention") op.kind = OP_ATTN;
            else if (l.kind == "layernorm") op.kind = OP_LN;
            else if (l.kind == "moe") op.kind = OP_MOE;
            else if (l.kind == "dropout") {
                op.kind = OP_DROPOUT;
                op.drop_rate = (float)std::stod(l.gets("rate", "0"));
                int site = 0;
                for (const Op& o : m->ops) site += o.kind == OP_DROPOUT ? 1 : 0;
                op.drop_site = site;
            }
            for (size_t wi = 0; wi < s.weights.size(); wi++)
                if (s.weights[wi].layer == op.layer) {
                    op.widx = (int)wi;
                    break;
                }
        }
        op.ints = so.ints;
        op.in = find_val(m, so.args[0]);
        if (so.args.size() > 1) op.in2 = find_val(m, so.args[1]);
        if (find_val(m, so.out) >= 0) {
            err = "value " + so.out + " assigned twice";
            return false;
        }
        Val v;
        v.name = so.out;
        v.cols = s.width[so.out];
        v.producer = (int)m->ops.size();
        m->vals.push_back(v);
        op.out = op.self_out = (int)m->vals.size() - 1;
        m->vals[op.in].consumers.push_back((int)m->ops.size());
        if (op.in2 >= 0) m->vals[op.in2].consumers.push_back((int)m->ops.size());
        m->ops.push_back(op);
    }
    m->out_val = find_val(m, s.output);
    // Fold `add(dense_or_attention_out, r)` into the producer's epilogue when
    // the product has no other consumer and no activation.
    for (size_t i = 0; i < m->ops.size(); i++) {
        Op& a = m->ops[i];
        if (a.kind != OP_ADD) continue;
        for (int side = 0; side < 2; side++) {
            int pv = side == 0 ? a.in : a.in2;
            int rv = side == 0 ? a.in2 : a.in;
            int pi = m->vals[pv].producer;
            if (pi < 0) continue;
            Op& p = m->ops[pi];
            if (!(p.kind == OP_DENSE && p.act == 0) && p.kind != OP_ATTN) continue;
            if (m->vals[pv].consumers.size() != 1 || pv == m->out_val) continue;
            if (m->vals[rv].producer >= pi) continue;  // residual must exist already
            if (pv == rv) continue;
            p.out = a.out;
            p.fused_res = rv;
            m->vals[pv].materialized = false;
            m->vals[a.out].producer = pi;
            a.skip = true;
            break;
        }
    }
    // A dropout of rate 0 is the identity in training too: its value shares
    // its input's storage. Others keep their own buffer (masked in training,
    // a copy in inference).
    for (auto& op : m->ops)
        if (op.kind == OP_DROPOUT && op.drop_rate == 0.f) m->vals[op.out].alias_of = op.in;
    // LayerNorm over a residual sum that a Dense (no activation) or attention
    // GEMM produces, 512 wide, the sum feeding nothing else: the GEMM can
    // normalise whole rows in its epilogue (a 128 x 512 tile holds them)
    for (size_t li = 0; li < m->ops.size(); li++) {
        Op& l = m->ops[li];
        if (l.kind != OP_LN) continue;
        const Val& r = m->vals[l.in];
        if (r.producer < 0 || r.cols != 512 || r.consumers.size() != 1 || l.in == m->out_val) continue;
        Op& p = m->ops[r.producer];
        if (p.skip || p.out != l.in || p.fused_res < 0 || p.ln_op >= 0) continue;
        if (!((p.kind == OP_DENSE && p.act == 0) || p.kind == OP_ATTN)) continue;
        p.ln_op = (int)li;
        l.ln_from = r.producer;
    }
    return true;
}

// Which forms each value must be stored in.
static void decide_storage(ns_model* m) {
    const bool bf = m->precision == 2;
    // LayerNorm fusion runs on the tensor-core path (TF32 / bf16 modes);
    // NS_B200_LN_FUSION=0 keeps the separate LayerNorm kernels
    const char* lf = getenv("NS_B200_LN_FUSION");
    m->ln_fusion = m->precision != 0 && !(lf && lf[0] == '0');
    for (auto& v : m->vals) v.ln_hidden = false;
    for (size_t vi = 0; vi < m->vals.size(); vi++) {
        Val& v = m->vals[vi];
        v.need_f32 = (int)vi == m->out_val || vi == 0;
        v.need_h16 = false;
        for (int ci : v.consumers) {
            const Op& c = m->ops[ci];
            if (c.skip) {
                // consumed as the residual of a fused add
                v.need_f32 = true;
                continue;
            }
            bool gemm_in = (c.kind == OP_DENSE || c.kind == OP_ATTN) && c.in == (int)vi;
            if (gemm_in && bf) v.need_h16 = true;
            else v.need_f32 = true;
            if (c.kind == OP_DENSE || c.kind == OP_ATTN || c.kind == OP_MOE) {
                if (c.fused_res == (int)vi) v.need_f32 = true;
            }
        }
        // a fused producer's residual operand is read in fp32
    }
    for (auto& op : m->ops)
        if (!op.skip && op.fused_res >= 0) m->vals[op.fused_res].need_f32 = true;
    // MoE reads its input in fp32 (exact router) and, in bf16 mode, in bf16
    for (auto& op : m->ops)
        if (op.kind == OP_MOE) {
            m->vals[op.in].need_f32 = true;
            if (bf) m->vals[op.in].need_h16 = true;
        }
    if (m->ln_fusion)
        for (auto& op : m->ops)
            if (op.ln_from >= 0) {
                // the sum is normalised in the producer's epilogue; the
                // backward works from the LayerNorm output (kept in fp32)
                m->vals[op.in].ln_hidden = true;
                m->vals[op.out].need_f32 = true;
            }
}

// ---------------------------------------------------------------------------
// working copies of the weights (GEMM operand dtype / packing)
// ---------------------------------------------------------------------------
static void free_working(ns_model* m) {
    for (size_t i = 0; i < m->wk.size(); i++)
        if (m->wk_owned[i] && m->wk[i]) cudaFree(m->wk[i]);
    m->wk.assign(m->spec.weights.size(), nullptr);
    m->wk_owned.assign(m->spec.weights.size(), false);
}

static int alloc_working(ns_model* m) {
    free_working(m);
    const Spec& s = m->spec;
    const bool bf = m->precision == 2;
    const size_t es = bf ? 2 : 4;
    for (size_t li = 0; li < s.layers.size(); li++) {
        const LayerSpec& l = s.layers[li];
        int w0 = -1;
        for (size_t wi = 0; wi < s.weights.size(); wi++)
            if (s.weights[wi].layer == (int)li) {
                w0 = (int)wi;
                break;
            }
        if (w0 < 0) continue;
        auto own = [&](int wi, size_t count) -> bool {
            void* p = persist_alloc(count * es);
            if (!p) return false;
            m->wk[wi] = p;
            m->wk_owned[wi] = true;
            return true;
        };
        auto alias_or_own = [&](int wi) -> bool {
            if (!bf) {
                m->wk[wi] = m->d_w + s.weights[wi].off;
                return true;
            }
            return own(wi, s.weights[wi].count);
        };
        if (l.kind == "dense") {
            if (!alias_or_own(w0)) return -1;
        } else if (l.kind == "attention") {
            long long d = l.geti("dim", 0);
            if (!own(w0, (size_t)3 * d * d)) return -1;  // packed [D, 3D] q|k|v
            if (!alias_or_own(w0 + 3)) return -1;        // o
        } else if (l.kind == "moe") {
            // router stays fp32 (read from the master blob); experts in the GEMM dtype
            if (!alias_or_own(w0 + 1)) return -1;
            if (l.gets("expert", "ffn") != "linear" && !alias_or_own(w0 + 2)) return -1;
        }
    }
    return 0;
}

// Where weight wi's working copy lives (dst == nullptr: the GEMMs read the
// fp32 master directly): a [rows, cols] view written at dst[r * ld + off + c].
struct WkTarget {
    void* dst = nullptr;
    long long ld = 0;
    int off = 0;
    int rows = 1, cols = 0;
};

static WkTarget working_target(const ns_model* m, int wi) {
    const Spec& s = m->spec;
    const WeightInfo& w = s.weights[wi];
    WkTarget t;
    if (w.layer < 0) return t;
    const LayerSpec& l = s.layers[w.layer];
    int w0 = wi;
    while (w0 > 0 && s.weights[w0 - 1].layer == w.layer) w0--;
    if (l.kind == "attention" && wi - w0 < 3) {
        const int d = (int)l.geti("dim", 0);
        t.dst = m->wk[w0];
        t.ld = 3LL * d;
        t.off = (wi - w0) * d;
        t.rows = d;
        t.cols = d;
        return t;
    }
    if (l.kind != "dense" && l.kind != "attention" && l.kind != "moe") return t;
    if (l.kind == "moe" && (wi == w0 || (wi == w0 + 2 && l.gets("expert", "ffn") == "linear"))) return t;
    if (!m->wk_owned[wi]) return t;
    t.dst = m->wk[wi];
    t.ld = (long long)w.count;
    t.rows = 1;
    t.cols = (int)w.count;
    return t;
}

// Refresh the working copies from the fp32 master blob (all of them, or
// those not marked in `done`).
static int refresh_working(ns_model* m, const std::vector<char>* done) {
    const Spec& s = m->spec;
    for (size_t wi = 0; wi < s.weights.size(); wi++) {
        if (done && (*done)[wi]) continue;
        const WkTarget t = working_target(m, (int)wi);
        if (!t.dst) continue;
        launch_counter() += 1;
        if (pack_weight(m->d_w + s.weights[wi].off, t.rows, t.cols, t.dst, m->wdt, t.ld, t.off, m->stream)) return -1;
    }
    return 0;
}

// The output layer can take the head GEMM + cross-entropy fusion: bf16
// tensor cores, cross-entropy loss, output straight from a Dense layer
// without activation or fused residual, at least 256 classes.
static const Op* ce_fusable_producer(const ns_model* m) {
    if (m->wdt != kBF16 || m->spec.loss == "mse" || m->out_val < 0) return nullptr;
    const Val& o = m->vals[m->out_val];
    if (o.producer < 0) return nullptr;
    const Op* p = &m->ops[o.producer];
    if (p->kind != OP_DENSE || p->act || p->fused_res >= 0 || p->skip || p->out != m->out_val) return nullptr;
    if (o.cols < 256 || o.cols % 8) return nullptr;
    return p;
}

// ---------------------------------------------------------------------------
// planning
// ---------------------------------------------------------------------------
static void free_plan(ns_model* m) {
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->wstream) cudaStreamSynchronize(m->wstream);
    for (void* p : m->plan_allocs) cudaFree(p);
    m->plan_allocs.clear();
    for (auto& v : m->vals) {
        v.f32 = nullptr;
        v.h16 = nullptr;
        v.gbuf = nullptr;
        v.gcur = nullptr;
    }
    for (auto& op : m->ops) {
        op.z = op.dz = op.qkv = op.ctx = op.dqkv = op.dctx = op.dout_w = nullptr;
        op.dz32 = op.lse = op.dvec = nullptr;
        op.ln_rstd = nullptr;
        moe_release(op);
    }
    m->d_in = m->d_labels = m->d_rowloss = m->d_loss = nullptr;
    m->d_targets = nullptr;
    m->d_stage = nullptr;
    m->d_ws = nullptr;
    m->d_ws2 = nullptr;
    m->ws2_floats = 0;
    m->ws_floats = 0;
    m->d_scratch = nullptr;
    m->scratch_bytes = 0;
    m->d_tlogit = nullptr;
    m->mmax = 0;
    m->train_planned = false;
}

#define PA(T, n) reinterpret_cast<T*>(plan_alloc(m, sizeof(T) * (size_t)(n)))

static int plan(ns_model* m, int M, bool train) {
    if (M <= m->mmax && (!train || m->train_planned)) return 0;
    int want = M > m->mmax ? M : m->mmax;
    want = (want + 127) / 128 * 128;
    free_plan(m);
    m->mmax = want;
    const size_t R = (size_t)want;
    const bool bf = m->precision == 2;
    const size_t es = bf ? 2 : 4;
    const Spec& s = m->spec;
    decide_storage(m);
    m->d_in = PA(float, R * s.in_cols);
    if (!m->d_in) return fail("device allocation failed");
    for (size_t vi = 1; vi < m->vals.size(); vi++) {
        Val& v = m->vals[vi];
        if (!v.materialized || v.alias_of >= 0 || v.ln_hidden) continue;
        if (v.need_f32) v.f32 = PA(float, R * v.cols);
        if (v.need_h16) v.h16 = PA(__nv_bfloat16, R * v.cols);
    }
    if (m->ln_fusion)
        for (auto& op : m->ops)
            if (op.ln_op >= 0) op.ln_rstd = PA(float, R);
    m->vals[0].f32 = m->d_in;
    if (m->vals[0].need_h16) m->vals[0].h16 = PA(__nv_bfloat16, R * s.in_cols);
    for (size_t vi = 1; vi < m->vals.size(); vi++) {
        Val& v = m->vals[vi];
        if (v.alias_of >= 0) {
            int a = v.alias_of;
            while (m->vals[a].alias_of >= 0) a = m->vals[a].alias_of;
            v.f32 = m->vals[a].f32;
            v.h16 = m->vals[a].h16;
        }
    }
    for (auto& op : m->ops) {
        if (op.skip) continue;
        const int cols = m->vals[op.self_out].cols;
        if (op.kind == OP_DENSE) {
            if (train && op.act) op.z = plan_alloc(m, R * cols * es);
            if (train) {
                if (bf) op.dz = plan_alloc(m, R * cols * 2);
                else if (op.act) op.dz32 = PA(float, R * cols);
            }
        } else if (op.kind == OP_ATTN) {
            const LayerSpec& l = s.layers[op.layer];
            int d = (int)l.geti("dim", 0), h = (int)l.geti("heads", 1);
            op.qkv = plan_alloc(m, R * 3 * d * es);
            op.ctx = plan_alloc(m, R * d * es);
            op.lse = PA(float, R * h);
            if (train) {
                op.dvec = PA(float, R * h);
                op.dqkv = plan_alloc(m, R * 3 * d * es);
                op.dctx = plan_alloc(m, R * d * es);
                if (bf) op.dout_w = plan_alloc(m, R * d * 2);
            }
        } else if (op.kind == OP_MOE) {
            if (moe_plan(m, op, want, train)) return fail("MoE plan failed: " + g_err);
        }
    }
    m->d_rowloss = PA(float, R);
    m->d_loss = PA(float, 4);
    if (train) {
        m->d_labels = PA(float, R * s.out_cols);
        m->d_targets = PA(int, R);
        for (size_t vi = 1; vi < m->vals.size(); vi++) {
            Val& v = m->vals[vi];
            v.gbuf = PA(float, R * v.cols);
        }
        // `grad input`: the network input's gradient is formed too
        if (s.input_grad) m->vals[0].gbuf = PA(float, R * s.in_cols);
        for (auto& op : m->ops)
            if (op.kind == OP_EMB) {
                const LayerSpec& l = s.layers[op.layer];
                size_t b = embedding_bwd_scratch_bytes(want, (int)l.geti("vocab", 1));
                if (b > m->scratch_bytes) m->scratch_bytes = b;
            }
        if (m->scratch_bytes) m->d_scratch = plan_alloc(m, m->scratch_bytes);
        if (ce_fusable_producer(m)) m->d_tlogit = PA(float, R);
        m->train_planned = true;
    }
    for (void* p : m->plan_allocs)
        if (!p) return fail("device allocation failed");
    return 0;
}

// split-K workspace on demand (sized once per plan)
static int run_gemm(ns_model* m, GemmDesc& d) {
    if (m->precision == 0) d.engine = kEngineSimt;
    size_t need = gemm_workspace_floats(d);
    if (need > m->ws_floats) {
        cudaStreamSynchronize(m->stream);
        void* p = plan_alloc(m, need * sizeof(float));
        if (!p) return fail("workspace allocation failed");
        m->d_ws = reinterpret_cast<float*>(p);
        m->ws_floats = need;
    }
    d.workspace = m->d_ws;
    d.workspace_floats = m->ws_floats;
    launch_counter() += gemm_uses_tensor_cores(d) && need ? 2 : 1;
    int r = gemm(d, m->stream, m->d_err);
    if (r) return fail("gemm launch failed (code " + std::to_string(r) + ")");
    return 0;
}

// A weight-gradient GEMM: on the side stream when this backward uses it
// (after everything issued so far on the main stream), else as run_gemm.
static int run_gemm_w(ns_model* m, GemmDesc& d) {
    if (!m->side_w) return run_gemm(m, d);
    size_t need = gemm_workspace_floats(d);
    if (need > m->ws2_floats) {
        cudaStreamSynchronize(m->wstream);
        void* p = plan_alloc(m, need * sizeof(float));
        if (!p) return fail("workspace allocation failed");
        m->d_ws2 = reinterpret_cast<float*>(p);
        m->ws2_floats = need;
    }
    d.workspace = m->d_ws2;
    d.workspace_floats = m->ws2_floats;
    cudaEventRecord(m->ev_ms, m->stream);
    cudaStreamWaitEvent(m->wstream, m->ev_ms, 0);
    launch_counter() += gemm_uses_tensor_cores(d) && need ? 2 : 1;
    int r = gemm(d, m->wstream, m->d_err);
    if (r) return fail("gemm launch failed (code " + std::to_string(r) + ")");
    m->side_used = true;
    return 0;
}

static GemmOperand opnd(const void* p, int dt, long long ld, bool mn) {
    GemmOperand o;
    o.ptr = p;
    o.dtype = dt;
    o.ld = ld;
    o.mn_major = mn;
    return o;
}

// the value's storage in the GEMM operand dtype
static const void* as_operand(ns_model* m, const Val& v) { return m->wdt == kBF16 ? (const void*)v.h16 : (const void*)v.f32; }

// ---------------------------------------------------------------------------
// region timing (events on the engine stream; read back after a sync)
// ---------------------------------------------------------------------------
static int region_begin(ns_model* m, const std::string& label) {
    if (!m->timing) return -1;
    int idx = -1;
    for (size_t i = 0; i < m->regions.size(); i++)
        if (m->regions[i].label == label) idx = (int)i;
    if (idx < 0) {
        m->regions.push_back(ns_model::Region());
        m->regions.back().label = label;
        idx = (int)m->regions.size() - 1;
    }
    ns_model::Region& r = m->regions[idx];
    std::pair<cudaEvent_t, cudaEvent_t> ev;
    if (!r.pool.empty()) {
        ev = r.pool.back();
        r.pool.pop_back();
    } else {
        cudaEventCreate(&ev.first);
        cudaEventCreate(&ev.second);
    }
    cudaEventRecord(ev.first, m->stream);
    r.pending.push_back(ev);
    return idx;
}

static void region_end(ns_model* m, int idx) {
    if (idx < 0) return;
    cudaEventRecord(m->regions[idx].pending.back().second, m->stream);
}

int nsb::region_open(ns_model* m, const std::string& label) { return region_begin(m, label); }
void nsb::region_close(ns_model* m, int idx) { region_end(m, idx); }

// A host-measured interval (e.g. time spent waiting on NCCL), folded into the
// same per-region totals.
static void host_region_add(ns_model* m, const char* label, double ms) {
    if (!m->timing) return;
    for (auto& r : m->regions)
        if (r.label == label) {
            r.ms += ms;
            r.count++;
            return;
        }
    m->regions.push_back(ns_model::Region());
    m->regions.back().label = label;
    m->regions.back().ms = ms;
    m->regions.back().count = 1;
}

static void regions_collect(ns_model* m) {
    for (auto& r : m->regions) {
        for (auto& ev : r.pending) {
            float ms = 0.f;
            if (cudaEventSynchronize(ev.second) == cudaSuccess && cudaEventElapsedTime(&ms, ev.first, ev.second) == cudaSuccess) {
                r.ms += ms;
                r.count++;
            }
            r.pool.push_back(ev);
        }
        r.pending.clear();
    }
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
static int forward(ns_model* m, int M, bool train) {
    const Spec& s = m->spec;
    if (m->vals[0].h16) {  // the raw input feeds a bf16 GEMM
        launch_counter() += 1;
        if (f32_to_bf16(m->d_in, (size_t)M * s.in_cols, m->vals[0].h16, m->stream)) return fail("input cast failed");
    }
    for (size_t oi = 0; oi < m->ops.size(); oi++) {
        Op& op = m->ops[oi];
        if (op.skip) continue;
        if (m->ln_fusion && op.ln_from >= 0) continue;  // normalised by its producer's GEMM
        Val& in = m->vals[op.in];
        Val& out = m->vals[op.out];
        int rc = 0;
        const std::string& lname = op.layer >= 0 ? s.layers[op.layer].name : s.ops[oi].out;
        int reg = op.kind == OP_ATTN ? -1 : region_begin(m, std::string("fwd:") + lname);
        switch (op.kind) {
            case OP_DENSE: {
                const WeightInfo& w = s.weights[op.widx];
                GemmDesc d;
                d.M = M;
                d.N = w.cols;
                d.K = w.rows;
                d.a = opnd(as_operand(m, in), m->wdt, w.rows, false);
                d.b = opnd(m->wk[op.widx], m->wdt, w.cols, true);
                d.ep.act = op.act;
                if (train && op.act) {
                    d.ep.z = op.z;
                    d.ep.z_dtype = m->wdt;
                    d.ep.ld_z = w.cols;
                }
                if (op.fused_res >= 0) {
                    d.ep.add = m->vals[op.fused_res].f32;
                    d.ep.ld_add = w.cols;
                }
                d.ep.c32 = out.f32;
                d.ep.ld_c32 = w.cols;
                d.ep.c16 = out.h16;
                d.ep.ld_c16 = w.cols;
                if (m->ln_fusion && op.ln_op >= 0) {
                    // the residual sum's LayerNorm in this GEMM's epilogue
                    const Val& n = m->vals[m->ops[op.ln_op].out];
                    d.ep.c32 = n.f32;
                    d.ep.c16 = n.h16;
                    d.ep.ln_rstd = op.ln_rstd;
                }
                if (train && m->ce_fused && op.out == m->out_val) {
                    // fp16 logits into the layer's gradient buffer (the loss
                    // pass turns them into the bf16 seed) and the target logits
                    d.ep.c32 = nullptr;
                    d.ep.c16 = reinterpret_cast<__nv_bfloat16*>(op.dz);
                    d.ep.c16_half = true;  // fp16 logits, overwritten by the bf16 seed
                    d.ep.ce_tgt = m->ce_targets;
                    d.ep.ce_tlogit = m->d_tlogit;
                }
                rc = run_gemm(m, d);
                break;
            }
            case OP_EMB: {
                const LayerSpec& l = s.layers[op.layer];
                const WeightInfo& w = s.weights[op.widx];
                launch_counter() += 1;
                rc = embedding_fwd(m->d_w + w.off, in.f32, M, (int)l.geti("vocab", 0), (int)l.geti("dim", 0), out.f32,
                                   out.h16, m->stream);
                break;
            }
            case OP_ATTN: {
                const LayerSpec& l = s.layers[op.layer];
                const int D = (int)l.geti("dim", 0), H = (int)l.geti("heads", 1);
                int S = (int)l.geti("seq", 0);
                if (S <= 0) S = M;
                if (M % S) return fail("attention: rows not a multiple of seq");
                GemmDesc d;
                d.M = M;
                d.N = 3 * D;
                d.K = D;
                d.a = opnd(as_operand(m, in), m->wdt, D, false);
                d.b = opnd(m->wk[op.widx], m->wdt, 3LL * D, true);
                if (m->wdt == kBF16) {
                    d.ep.c16 = reinterpret_cast<__nv_bfloat16*>(op.qkv);
                    d.ep.ld_c16 = 3 * D;
                } else {
                    d.ep.c32 = reinterpret_cast<float*>(op.qkv);
                    d.ep.ld_c32 = 3 * D;
                }
                int r1 = region_begin(m, "fwd:" + lname + ".qkv");
                rc = run_gemm(m, d);
                region_end(m, r1);
                if (rc) break;
                AttnArgs a;
                a.B = M / S;
                a.S = S;
                a.H = H;
                a.D = D;
                a.dh = D / H;
                a.scale = 1.0f / sqrtf((float)(D / H));
                a.dtype = m->wdt;
                a.qkv = op.qkv;
                a.ld_qkv = 3LL * D;
                a.ctx = op.ctx;
                a.ld_ctx = D;
                a.lse = op.lse;
                a.err = m->d_err;
                launch_counter() += 1;
                int r2 = region_begin(m, "fwd:" + lname + ".core");
                rc = attention_fwd(a, m->stream);
                region_end(m, r2);
                if (rc) {
                    rc = fail("attention launch failed");
                    break;
                }
                GemmDesc o;
                o.M = M;
                o.N = D;
                o.K = D;
                o.a = opnd(op.ctx, m->wdt, D, false);
                o.b = opnd(m->wk[op.widx + 3], m->wdt, D, true);
                if (op.fused_res >= 0) {
                    o.ep.add = m->vals[op.fused_res].f32;
                    o.ep.ld_add = D;
                }
                o.ep.c32 = out.f32;
                o.ep.ld_c32 = D;
                o.ep.c16 = out.h16;
                o.ep.ld_c16 = D;
                if (m->ln_fusion && op.ln_op >= 0) {
                    const Val& n = m->vals[m->ops[op.ln_op].out];
                    o.ep.c32 = n.f32;
                    o.ep.c16 = n.h16;
                    o.ep.ln_rstd = op.ln_rstd;
                }
                int r3 = region_begin(m, "fwd:" + lname + ".out");
                rc = run_gemm(m, o);
                region_end(m, r3);
                break;
            }
            case OP_LN:
                launch_counter() += 1;
                rc = layernorm_fwd(in.f32, M, in.cols, out.f32, out.h16, m->stream);
                break;
            case OP_ADD:
            case OP_SUB:
            case OP_MUL:
            case OP_DIV:
                launch_counter() += 1;
                rc = binop_fwd(in.f32, m->vals[op.in2].f32, (size_t)M * in.cols, op.kind - OP_ADD, out.f32, out.h16,
                               m->stream);
                break;
            case OP_CONCAT:
                launch_counter() += 1;
                rc = concat_cols(in.f32, in.cols, m->vals[op.in2].f32, m->vals[op.in2].cols, M, out.f32, out.h16,
                                 m->stream);
                break;
            case OP_SLICE:
                launch_counter() += 1;
                rc = slice_cols(in.f32, M, in.cols, (int)op.ints[0], (int)op.ints[1], out.f32, out.h16, m->stream);
                break;
            case OP_INDEX:
                launch_counter() += 1;
                rc = index_cols(in.f32, M, in.cols, op.d_idx, (int)op.ints.size(), out.f32, out.h16, m->stream);
                break;
            case OP_SCATTER:
                launch_counter() += 1;
                rc = scatter_cols(in.f32, M, in.cols, op.d_idx, (int)op.ints.size(), m->vals[op.in2].f32, out.f32,
                                  out.h16, m->stream);
                break;
            case OP_ACT:
                launch_counter() += 1;
                rc = act_fwd_f32(in.f32, (size_t)M * in.cols, op.act, out.f32, out.h16, m->stream);
                break;
            case OP_SOFTMAX:
                launch_counter() += 1;
                rc = softmax_rows(in.f32, M, in.cols, out.f32, out.h16, m->stream);
                break;
            case OP_DROPOUT: {
                if (op.drop_rate == 0.f) break;  // identity, storage shared with the input
                DropoutSite d;
                d.rate = train ? op.drop_rate : 0.f;  // inference: a copy
                d.key0 = m->drop_key0;
                d.key1 = m->drop_key1;
                d.step = m->drop_step;
                d.site = (uint32_t)op.drop_site;
                // data parallel: this rank's rows follow rank x M rows of the batch
                d.base = (unsigned long long)m->rank * (unsigned long long)M * (unsigned long long)in.cols;
                launch_counter() += 1;
                rc = dropout_fwd(in.f32, (size_t)M * in.cols, d, out.f32, out.h16, m->stream);
                break;
            }
            case OP_MOE:
                rc = moe_forward(m, op, M, train);
                break;
            default:
                return fail("operation not supported by this backend: " + s.ops[oi].fn);
        }
        region_end(m, reg);
        if (rc) return rc < 0 && !g_err.empty() ? -1 : fail("kernel launch failed in " + s.ops[oi].out);
    }
    return 0;
}

// ---------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------
// Add an existing gradient buffer `src` into value v's running total.
static int contribute_alias(ns_model* m, Val& v, const float* src, int M) {
    if (!v.gbuf) return 0;  // input x / non-differentiable
    if (!v.gcur) {
        v.gcur = src;
        return 0;
    }
    launch_counter() += 1;
    int rc = add_f32(v.gcur, src, (size_t)M * v.cols, v.gbuf, nullptr, m->stream);
    v.gcur = v.gbuf;
    return rc;
}

// gradient (fp32) of a value -> GEMM operand dtype buffer
static const void* grad_operand(ns_model* m, const float* g, void* tmp16, size_t n) {
    if (m->wdt != kBF16) return g;
    launch_counter() += 1;
    f32_to_bf16(g, n, reinterpret_cast<__nv_bfloat16*>(tmp16), m->stream);
    return tmp16;
}

// ---------------------------------------------------------------------------
// data-parallel gradient reduction, overlapped with the backward pass: as a
// layer's weight gradients are complete, their blob range is all-reduced on
// the communication stream while the backward of earlier layers continues.
// All ranks issue the same ranges in the same (reverse layer) order.
// ---------------------------------------------------------------------------
static int nccl_settle(ns_model* m);
static int optimizer_step(ns_model* m, float lr, const std::vector<char>* sel = nullptr);
static int refresh_working(ns_model* m, const std::vector<char>* done);
void assign_owners(ns_model* m);
static bool dist_active(const ns_model* m) { return m->comm && m->world > 1; }

static cudaEvent_t dist_event(ns_model* m) {
    if (m->ev_next >= m->dist_events.size()) {
        cudaEvent_t e = nullptr;
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return nullptr;
        m->dist_events.push_back(e);
    }
    return m->dist_events[m->ev_next++];
}

// One collective on the communication stream, ordered after the work so
// far on the engine stream: all-reduce (root < 0) or reduce to `root` of the
// gradient range, or (bcast) broadcast of the weight range from `root`.
static int dist_collective(ns_model* m, size_t off, size_t count, int root, bool bcast) {
    if (!count) return 0;
    cudaEvent_t ev = dist_event(m);
    if (!ev) return fail("event creation failed");
    cudaEventRecord(ev, m->stream);
    cudaStreamWaitEvent(m->comm_stream, ev, 0);
    if (m->side_w && m->side_used) {
        // weight gradients computed on the backward's second stream: the
        // collective also follows everything issued there so far
        cudaEvent_t ev2 = dist_event(m);
        if (!ev2) return fail("event creation failed");
        cudaEventRecord(ev2, m->wstream);
        cudaStreamWaitEvent(m->comm_stream, ev2, 0);
    }
    launch_counter() += 1;
    ncclResult_t r;
    if (bcast)
        r = nccl().Broadcast(m->d_w + off, m->d_w + off, count, ncclFloat, root, m->comm, m->comm_stream);
    else if (root >= 0)
        r = nccl().Reduce(m->d_g + off, m->d_g + off, count, ncclFloat, ncclSum, root, m->comm, m->comm_stream);
    else
        r = nccl().AllReduce(m->d_g + off, m->d_g + off, count, ncclFloat, ncclSum, m->comm, m->comm_stream);
    if (r != ncclSuccess && r != ncclInProgress) return fail(std::string("collective: ") + nccl().GetErrorString(r));
    // a non-blocking communicator may still be enqueueing: wait until the
    // collective sits on its stream before the next NCCL call
    if (r == ncclInProgress && nccl_settle(m)) return -1;
    cudaEvent_t after = dist_event(m);
    if (!after) return fail("event creation failed");
    cudaEventRecord(after, m->comm_stream);
    m->bucket_done.push_back(after);
    return 0;
}

static int dist_reduce_range(ns_model* m, size_t off, size_t count) { return dist_collective(m, off, count, -1, false); }

// Reduce the gradients of weights [w0, w1) once they are final: matrices
// with an owner rank (sharded Muon) are reduced to their owner only, the
// rest all-reduced in contiguous runs; the loss sum stored after the blob
// rides with an all-reduce that ends the blob, or alone.
static int dist_reduce_weights(ns_model* m, int w0, int w1) {
    const Spec& s = m->spec;
    for (int w = w0; w < w1; w++)
        if (m->reduced[w]) return 0;
    for (int w = w0; w < w1; w++) m->reduced[w] = 1;
    m->bucket_w.push_back(std::make_pair(w0, w1));
    const size_t ev0 = m->bucket_done.size();
    int w = w0;
    while (w < w1) {
        const int own = m->owner.empty() ? -1 : m->owner[w];
        if (own >= 0) {
            if (dist_collective(m, s.weights[w].off, s.weights[w].count, own, false)) return -1;
            if (s.weights[w].off + s.weights[w].count == s.total && dist_reduce_range(m, s.total, 1)) return -1;
            w++;
            continue;
        }
        int e = w;
        while (e < w1 && (m->owner.empty() || m->owner[e] < 0)) e++;
        const size_t off = s.weights[w].off;
        size_t end = s.weights[e - 1].off + s.weights[e - 1].count;
        if (end == s.total) end += 1;
        if (dist_reduce_range(m, off, end - off)) return -1;
        w = e;
    }
    // completion of the bucket = completion of its last collective
    m->bucket_evt.push_back(m->bucket_done.size() > ev0 ? m->bucket_done.back() : nullptr);
    return 0;
}

// Reduce what is left (weights of layers without a gradient op in this
// step, or layers applied more than once), then order the main stream after
// every reduction.
static int dist_reduce_finish(ns_model* m) {
    const Spec& s = m->spec;
    const int nw = (int)s.weights.size();
    int w = 0;
    while (w < nw) {
        if (m->reduced[w]) {
            w++;
            continue;
        }
        int e = w;
        while (e < nw && !m->reduced[e]) e++;
        if (dist_reduce_weights(m, w, e)) return -1;
        w = e;
    }
    if (nw == 0) {
        m->bucket_w.push_back(std::make_pair(0, 0));
        if (dist_reduce_range(m, s.total, 1)) return -1;
        m->bucket_evt.push_back(m->bucket_done.back());
    }
    return 0;
}

// Optimizer step under data parallelism: the weights of every bucket but the
// last are updated as soon as their all-reduces are done, while the last
// bucket (the first layer's gradients, finished last by the backward) is
// still being reduced; then the rest.
static int dist_optimizer(ns_model* m, float lr) {
    const size_t nb = m->bucket_w.size();
    const size_t nw = m->spec.weights.size();
    bool sharded = false;
    for (int o : m->owner) sharded = sharded || o >= 0;
    if (sharded) {
        // Sharded Muon: every reduction done; update the replicated (AdamW)
        // weights and the matrices this rank owns; broadcast each owned
        // matrix from its owner (weight order, the same on every rank); then
        // refresh the working copies of the matrices received.
        int ra = region_begin(m, "allreduce");
        if (!m->bucket_done.empty()) cudaStreamWaitEvent(m->stream, m->bucket_done.back(), 0);
        region_end(m, ra);
        std::vector<char> mine(nw, 0), received(nw, 1);
        for (size_t w = 0; w < nw; w++) {
            mine[w] = m->owner[w] < 0 || m->owner[w] == m->rank;
            if (m->owner[w] >= 0 && m->owner[w] != m->rank) received[w] = 0;
        }
        int ro = region_begin(m, "optimizer");
        if (optimizer_step(m, lr, &mine)) return -1;
        region_end(m, ro);
        int rb = region_begin(m, "broadcast");
        const size_t before = m->bucket_done.size();
        for (size_t w = 0; w < nw; w++)
            if (m->owner[w] >= 0 &&
                dist_collective(m, m->spec.weights[w].off, m->spec.weights[w].count, m->owner[w], true))
                return -1;
        if (m->bucket_done.size() > before) cudaStreamWaitEvent(m->stream, m->bucket_done.back(), 0);
        region_end(m, rb);
        return refresh_working(m, &received);
    }
    if (nb >= 2) {
        std::vector<char> early(nw, 0);
        for (size_t b = 0; b + 1 < nb; b++)
            for (int w = m->bucket_w[b].first; w < m->bucket_w[b].second; w++) early[w] = 1;
        // (collectives complete in issue order on the one communication stream)
        if (m->bucket_evt[nb - 2]) cudaStreamWaitEvent(m->stream, m->bucket_evt[nb - 2], 0);
        int ro = region_begin(m, "optimizer");
        if (optimizer_step(m, lr, &early)) return -1;
        region_end(m, ro);
        int ra = region_begin(m, "allreduce");  // what is left to wait for
        cudaStreamWaitEvent(m->stream, m->bucket_done.back(), 0);
        region_end(m, ra);
        std::vector<char> late(nw, 0);
        for (size_t w = 0; w < nw; w++) late[w] = !early[w];
        int rl = region_begin(m, "optimizer.last");
        if (optimizer_step(m, lr, &late)) return -1;
        region_end(m, rl);
        return 0;
    }
    int ra = region_begin(m, "allreduce");
    if (!m->bucket_done.empty()) cudaStreamWaitEvent(m->stream, m->bucket_done.back(), 0);
    region_end(m, ra);
    int ro = region_begin(m, "optimizer");
    if (optimizer_step(m, lr)) return -1;
    region_end(m, ro);
    return 0;
}

// Weight index range [w0, w1) of a layer (w0 == w1: none).
static void layer_weights(const ns_model* m, int layer, int& w0, int& w1) {
    const Spec& s = m->spec;
    w0 = w1 = -1;
    for (size_t wi = 0; wi < s.weights.size(); wi++)
        if (s.weights[wi].layer == layer) {
            if (w0 < 0) w0 = (int)wi;
            w1 = (int)wi + 1;
        }
    if (w0 < 0) w0 = w1 = 0;
}

static int backward_ops(ns_model* m, int M);

static int backward(ns_model* m, int M) {
    // weight gradients on the side stream: bf16 (every dW GEMM reads a bf16
    // operand buffer of its own op), not while regions are timed; under data
    // parallelism each bucket's collective also waits for the side stream
    m->side_w = m->wstream && m->wdt == kBF16 && !m->timing;
    m->side_used = false;
    m->emb_sorted = -1;
    if (m->side_w && m->d_scratch) {
        // a single embedding layer: its gradient's counting sort needs only
        // the ids, so it runs on the side stream while the backward starts
        int emb = -1, n_emb = 0;
        for (size_t oi = 0; oi < m->ops.size(); oi++)
            if (!m->ops[oi].skip && m->ops[oi].kind == OP_EMB) {
                emb = (int)oi;
                n_emb++;
            }
        if (n_emb == 1) {
            const Op& op = m->ops[emb];
            const LayerSpec& l = m->spec.layers[op.layer];
            cudaEventRecord(m->ev_ms, m->stream);  // the ids are on the device
            cudaStreamWaitEvent(m->wstream, m->ev_ms, 0);
            launch_counter() += 4;
            if (embedding_bwd_sort(m->vals[op.in].f32, M, (int)l.geti("vocab", 0), m->d_scratch, m->wstream))
                return fail("embedding sort launch failed");
            cudaEventRecord(m->ev_emb, m->wstream);
            m->side_used = true;
            m->emb_sorted = emb;
        }
    }
    const int rc = backward_ops(m, M);
    if (m->side_used) {  // the optimizer and the next step follow every dW GEMM
        cudaEventRecord(m->ev_sm, m->wstream);
        cudaStreamWaitEvent(m->stream, m->ev_sm, 0);
    }
    m->side_w = false;
    return rc;
}

static int backward_ops(ns_model* m, int M) {
    const Spec& s = m->spec;
    for (int oi = (int)m->ops.size() - 1; oi >= 0; oi--) {
        Op& op = m->ops[oi];
        if (op.skip) continue;
        Val& out = m->vals[op.out];
        if (!out.gcur) continue;
        const float* dv = out.gcur;
        Val& in = m->vals[op.in];
        int rc = 0;
        const std::string rname = std::string("bwd:") + (op.layer >= 0 ? s.layers[op.layer].name : s.ops[oi].out);
        const int reg = op.kind == OP_ATTN ? -1 : region_begin(m, rname);
        switch (op.kind) {
            case OP_DENSE: {
                const WeightInfo& w = s.weights[op.widx];
                const size_t n = (size_t)M * w.cols;
                const void* dz;
                if (op.act && op.dz_ready) {
                    // the consumer's input-gradient GEMM already applied act'
                    dz = m->wdt == kBF16 ? op.dz : (const void*)op.dz32;
                    op.dz_ready = false;
                } else if (op.act) {
                    launch_counter() += 1;
                    if (m->wdt == kBF16) {
                        rc = act_bwd(dv, op.z, kBF16, op.act, nullptr, n, nullptr,
                                     reinterpret_cast<__nv_bfloat16*>(op.dz), m->stream);
                        dz = op.dz;
                    } else {
                        rc = act_bwd(dv, op.z, kF32, op.act, nullptr, n, op.dz32, nullptr, m->stream);
                        dz = op.dz32;
                    }
                    if (rc) break;
                } else if (m->seed16 && oi == m->vals[m->out_val].producer) {
                    dz = op.dz;  // the loss kernel wrote the bf16 seed here
                } else if (op.g16_ready) {
                    dz = op.dz;  // the consumer's LN backward wrote the bf16 copy
                    op.g16_ready = false;
                } else {
                    dz = grad_operand(m, dv, op.dz, n);
                }
                if (op.fused_res >= 0 && (rc = contribute_alias(m, m->vals[op.fused_res], dv, M))) break;
                GemmDesc gw;
                gw.M = w.rows;
                gw.N = w.cols;
                gw.K = M;
                gw.a = opnd(as_operand(m, in), m->wdt, w.rows, true);
                gw.b = opnd(dz, m->wdt, w.cols, true);
                gw.ep.c32 = m->d_g + w.off;
                gw.ep.ld_c32 = w.cols;
                if ((rc = run_gemm_w(m, gw))) break;
                if (in.gbuf) {
                    GemmDesc gx;
                    gx.M = M;
                    gx.N = w.rows;
                    gx.K = w.cols;
                    gx.a = opnd(dz, m->wdt, w.cols, false);
                    gx.b = opnd(m->wk[op.widx], m->wdt, w.cols, false);
                    // The input is a Dense layer's activation output consumed only
                    // here: apply that layer's act' in this epilogue and write its
                    // pre-activation gradient straight into its GEMM operand buffer.
                    Op* P = in.producer >= 0 ? &m->ops[in.producer] : nullptr;
                    if (P && !in.gcur && P->kind == OP_DENSE && P->act && !P->skip && P->self_out == op.in &&
                        P->fused_res < 0 && in.consumers.size() == 1 && P->z &&
                        (m->wdt == kBF16 ? P->dz != nullptr : P->dz32 != nullptr)) {
                        gx.ep.dz = P->z;
                        gx.ep.dz_dtype = m->wdt;
                        gx.ep.ld_dz = w.rows;
                        gx.ep.dz_act = P->act;
                        if (m->wdt == kBF16) {
                            gx.ep.c16 = reinterpret_cast<__nv_bfloat16*>(P->dz);
                            gx.ep.ld_c16 = w.rows;
                        } else {
                            gx.ep.c32 = P->dz32;
                            gx.ep.ld_c32 = w.rows;
                        }
                        if ((rc = run_gemm(m, gx))) break;
                        P->dz_ready = true;
                        in.gcur = in.gbuf;  // marks the gradient present; P reads its dz
                        break;
                    }
                    if (in.gcur) {
                        gx.ep.add = in.gcur;
                        gx.ep.ld_add = w.rows;
                    }
                    gx.ep.c32 = in.gbuf;
                    gx.ep.ld_c32 = w.rows;
                    if ((rc = run_gemm(m, gx))) break;
                    in.gcur = in.gbuf;
                }
                break;
            }
            case OP_EMB: {
                const LayerSpec& l = s.layers[op.layer];
                const WeightInfo& w = s.weights[op.widx];
                if (m->emb_sorted == oi) {  // the sort ran ahead on the side stream
                    cudaStreamWaitEvent(m->stream, m->ev_emb, 0);
                    launch_counter() += 2;
                    rc = embedding_bwd_sum(dv, M, (int)l.geti("vocab", 0), (int)l.geti("dim", 0), m->d_g + w.off,
                                           m->d_scratch, m->stream);
                } else {
                    launch_counter() += 5;
                    rc = embedding_bwd(dv, in.f32, M, (int)l.geti("vocab", 0), (int)l.geti("dim", 0),
                                       m->d_g + w.off, m->d_scratch, m->stream);
                }
                break;
            }
            case OP_ATTN: {
                const LayerSpec& l = s.layers[op.layer];
                const int D = (int)l.geti("dim", 0), H = (int)l.geti("heads", 1);
                int S = (int)l.geti("seq", 0);
                if (S <= 0) S = M;
                int r1 = region_begin(m, rname + ".out");
                const void* dout = op.g16_ready ? op.dout_w : grad_operand(m, dv, op.dout_w, (size_t)M * D);
                op.g16_ready = false;
                if (op.fused_res >= 0 && (rc = contribute_alias(m, m->vals[op.fused_res], dv, M))) break;
                const WeightInfo& wo = s.weights[op.widx + 3];
                GemmDesc go;  // dWo = ctx^T dout
                go.M = D;
                go.N = D;
                go.K = M;
                go.a = opnd(op.ctx, m->wdt, D, true);
                go.b = opnd(dout, m->wdt, D, true);
                go.ep.c32 = m->d_g + wo.off;
                go.ep.ld_c32 = D;
                if ((rc = run_gemm_w(m, go))) break;
                GemmDesc gc;  // dctx = dout Wo^T
                gc.M = M;
                gc.N = D;
                gc.K = D;
                gc.a = opnd(dout, m->wdt, D, false);
                gc.b = opnd(m->wk[op.widx + 3], m->wdt, D, false);
                if (m->wdt == kBF16) {
                    gc.ep.c16 = reinterpret_cast<__nv_bfloat16*>(op.dctx);
                    gc.ep.ld_c16 = D;
                } else {
                    gc.ep.c32 = reinterpret_cast<float*>(op.dctx);
                    gc.ep.ld_c32 = D;
                }
                if ((rc = run_gemm(m, gc))) break;
                region_end(m, r1);
                int r2 = region_begin(m, rname + ".core");
                AttnArgs a;
                a.B = M / S;
                a.S = S;
                a.H = H;
                a.D = D;
                a.dh = D / H;
                a.scale = 1.0f / sqrtf((float)(D / H));
                a.dtype = m->wdt;
                a.qkv = op.qkv;
                a.ld_qkv = 3LL * D;
                a.ctx = op.ctx;
                a.ld_ctx = D;
                a.lse = op.lse;
                a.dctx = op.dctx;
                a.ld_dctx = D;
                a.dqkv = op.dqkv;
                a.ld_dqkv = 3LL * D;
                a.dvec = op.dvec;
                a.err = m->d_err;
                launch_counter() += attention_bwd_launches(a);
                if ((rc = attention_bwd(a, m->stream))) {
                    rc = fail("attention backward launch failed");
                    break;
                }
                region_end(m, r2);
                int r3 = region_begin(m, rname + ".qkv");
                {  // [dWq | dWk | dWv] = x^T [dQ | dK | dV]: one GEMM, N = 3D, whose
                   // column blocks land on the three consecutive blob tensors
                    const WeightInfo& wq = s.weights[op.widx];
                    GemmDesc gq;
                    gq.M = D;
                    gq.N = 3 * D;
                    gq.K = M;
                    gq.a = opnd(as_operand(m, in), m->wdt, D, true);
                    gq.b = opnd(op.dqkv, m->wdt, 3LL * D, true);
                    gq.ep.c32 = m->d_g + wq.off;
                    gq.ep.ld_c32 = D;
                    gq.ep.col_block = D;
                    gq.ep.col_block_stride = (long long)D * D;
                    if ((rc = run_gemm_w(m, gq))) break;
                }
                if (in.gbuf) {
                    GemmDesc gx;  // dx = dQKV [Wq|Wk|Wv]^T (+ running total)
                    gx.M = M;
                    gx.N = D;
                    gx.K = 3 * D;
                    gx.a = opnd(op.dqkv, m->wdt, 3LL * D, false);
                    gx.b = opnd(m->wk[op.widx], m->wdt, 3LL * D, false);
                    if (in.gcur) {
                        gx.ep.add = in.gcur;
                        gx.ep.ld_add = D;
                    }
                    gx.ep.c32 = in.gbuf;
                    gx.ep.ld_c32 = D;
                    if ((rc = run_gemm(m, gx))) break;
                    in.gcur = in.gbuf;
                }
                region_end(m, r3);
                break;
            }
            case OP_LN: {
                if (!in.gbuf) break;
                // When the LN input comes straight from a Dense (no activation)
                // or Attention layer and LN is its only consumer, also write the
                // gradient as that layer's bf16 GEMM operand (saves a cast pass).
                __nv_bfloat16* dx16 = nullptr;
                Op* P = in.producer >= 0 ? &m->ops[in.producer] : nullptr;
                if (m->wdt == kBF16 && P && !P->skip && P->out == op.in && in.consumers.size() == 1) {
                    if (P->kind == OP_DENSE && P->act == 0 && P->dz) dx16 = reinterpret_cast<__nv_bfloat16*>(P->dz);
                    else if (P->kind == OP_ATTN && P->dout_w) dx16 = reinterpret_cast<__nv_bfloat16*>(P->dout_w);
                }
                launch_counter() += 1;
                if (m->ln_fusion && op.ln_from >= 0)  // from the output and the GEMM's rstd
                    rc = layernorm_bwd_from_output(dv, out.f32, m->ops[op.ln_from].ln_rstd, in.gcur, M, in.cols,
                                                   in.gbuf, dx16, m->stream);
                else
                    rc = layernorm_bwd(dv, in.f32, in.gcur, M, in.cols, in.gbuf, dx16, m->stream);
                in.gcur = in.gbuf;
                if (dx16) P->g16_ready = true;
                break;
            }
            case OP_ADD:
                if ((rc = contribute_alias(m, in, dv, M))) break;
                rc = contribute_alias(m, m->vals[op.in2], dv, M);
                break;
            case OP_ACT:
                if (!in.gbuf) break;
                launch_counter() += 1;
                rc = act_bwd(dv, in.f32, kF32, op.act, in.gcur, (size_t)M * in.cols, in.gbuf, nullptr, m->stream);
                in.gcur = in.gbuf;
                break;
            case OP_SUB:
            case OP_MUL:
            case OP_DIV: {
                // two passes (a then b) so that op(x, x) accumulates correctly
                Val& b = m->vals[op.in2];
                const size_t n = (size_t)M * in.cols;
                const int code = op.kind - OP_ADD;
                if (in.gbuf) {
                    launch_counter() += 1;
                    if ((rc = binop_bwd(dv, in.f32, b.f32, n, code, in.gcur, in.gbuf, nullptr, nullptr, m->stream))) break;
                    in.gcur = in.gbuf;
                }
                if (b.gbuf) {
                    launch_counter() += 1;
                    if ((rc = binop_bwd(dv, in.f32, b.f32, n, code, nullptr, nullptr, b.gcur, b.gbuf, m->stream))) break;
                    b.gcur = b.gbuf;
                }
                break;
            }
            case OP_CONCAT: {
                Val& b = m->vals[op.in2];
                if (in.gbuf) {
                    launch_counter() += 1;
                    if ((rc = concat_cols_bwd(dv, in.cols, b.cols, M, in.gcur, in.gbuf, nullptr, nullptr, m->stream)))
                        break;
                    in.gcur = in.gbuf;
                }
                if (b.gbuf) {
                    launch_counter() += 1;
                    if ((rc = concat_cols_bwd(dv, in.cols, b.cols, M, nullptr, nullptr, b.gcur, b.gbuf, m->stream)))
                        break;
                    b.gcur = b.gbuf;
                }
                break;
            }
            case OP_SLICE:
                if (!in.gbuf) break;
                launch_counter() += 1;
                rc = slice_cols_bwd(dv, M, in.cols, (int)op.ints[0], (int)op.ints[1], in.gcur, in.gbuf, m->stream);
                in.gcur = in.gbuf;
                break;
            case OP_INDEX:
                if (!in.gbuf) break;
                launch_counter() += 1;
                rc = index_cols_bwd(dv, M, in.cols, op.d_idx, (int)op.ints.size(), in.gcur, in.gbuf, m->stream);
                in.gcur = in.gbuf;
                break;
            case OP_SCATTER: {
                Val& u = m->vals[op.in2];
                const int L = (int)op.ints.size();
                if (in.gbuf) {
                    launch_counter() += 1;
                    if ((rc = scatter_cols_bwd(dv, M, in.cols, op.d_idx, L, in.gcur, in.gbuf, nullptr, nullptr,
                                               m->stream)))
                        break;
                    in.gcur = in.gbuf;
                }
                if (u.gbuf) {
                    launch_counter() += 2;
                    if ((rc = scatter_cols_bwd(dv, M, in.cols, op.d_idx, L, nullptr, nullptr, u.gcur, u.gbuf,
                                               m->stream)))
                        break;
                    u.gcur = u.gbuf;
                }
                break;
            }
            case OP_DROPOUT:
                if (op.drop_rate > 0.f) {
                    if (!in.gbuf) break;
                    DropoutSite d;
                    d.rate = op.drop_rate;
                    d.key0 = m->drop_key0;
                    d.key1 = m->drop_key1;
                    d.step = m->drop_step;
                    d.site = (uint32_t)op.drop_site;
                    d.base = (unsigned long long)m->rank * (unsigned long long)M * (unsigned long long)in.cols;
                    launch_counter() += 1;
                    rc = dropout_bwd(dv, (size_t)M * in.cols, d, in.gcur, in.gbuf, m->stream);
                    in.gcur = in.gbuf;
                    break;
                }
                rc = contribute_alias(m, in, dv, M);
                break;
            case OP_SOFTMAX:  // the reference's softmax gradient is a pass-through (code 0)
                rc = contribute_alias(m, in, dv, M);
                break;
            case OP_MOE:
                rc = moe_backward(m, op, M);
                break;
            default:
                return fail("backward not supported for " + s.ops[oi].fn);
        }
        region_end(m, reg);
        if (rc) return -1;
        if (dist_active(m) && op.layer >= 0) {
            // a layer applied by more than one op is reduced at the end
            int uses = 0;
            for (const Op& o2 : m->ops) uses += (!o2.skip && o2.layer == op.layer) ? 1 : 0;
            int w0, w1;
            layer_weights(m, op.layer, w0, w1);
            if (uses == 1 && w1 > w0 && dist_reduce_weights(m, w0, w1)) return -1;
        }
    }
    return 0;
}

// ---------------------------------------------------------------------------
// loss + optimizer
// ---------------------------------------------------------------------------
static float lr_schedule(const ns_model* m, long long step) {
    const Spec& s = m->spec;
    if (s.schedule != "cosine") return 1.0f;
    const long long warm = (long long)s.schedv("warmup", 100), total = (long long)s.schedv("total", 10000);
    const float minf = (float)s.schedv("min", 0.05);
    if (warm <= 0) return 1.0f;
    if (step < warm) return (float)step / (float)warm;
    const long long end = total > warm ? total : warm + 1;
    const long long st = step >= end ? end : step;
    const float t = (float)(st - warm) / (float)(end - warm);
    return minf + 0.5f * (1.0f - minf) * (1.0f + cosf(3.14159265f * t));
}

static int loss_and_seed(ns_model* m, int M, const float* labels, const int* targets, bool want_grad) {
    Val& o = m->vals[m->out_val];
    const int C = o.cols;
    const float denom = (float)M * (float)m->world;
    // When the output comes straight from a Dense layer without activation
    // or fused residual, its backward only needs the seed as a bf16 GEMM
    // operand: the loss kernel writes it there and skips the fp32 copy.
    const Op* prod = o.producer >= 0 ? &m->ops[o.producer] : nullptr;
    m->seed16 = want_grad && m->wdt == kBF16 && prod && prod->kind == OP_DENSE && prod->act == 0 &&
                prod->fused_res < 0 && prod->dz;
    float* d32 = want_grad && !m->seed16 ? o.gbuf : nullptr;
    __nv_bfloat16* d16 = m->seed16 ? reinterpret_cast<__nv_bfloat16*>(prod->dz) : nullptr;
    launch_counter() += 1;
    int rc;
    if (m->ce_fused) {
        rc = cross_entropy_finish(d16, M, C, targets, m->d_tlogit, denom, m->d_rowloss, m->stream);
    } else if (m->spec.loss == "mse") {
        if (!labels) return fail("mse loss needs dense targets");
        rc = mse_fwd_bwd(o.f32, labels, M, C, want_grad ? (float)M * C * m->world : 1.f, m->d_rowloss, d32, d16,
                         m->stream);
    } else {
        rc = cross_entropy_fwd_bwd(o.f32, labels, targets, M, C, denom, m->d_rowloss, d32, d16, m->stream);
    }
    if (rc) return fail("loss kernel launch failed");
    if (want_grad) o.gcur = o.gbuf;
    return 0;
}

struct AdamTensorLocal {
    float* w;
    const float* g;
    float* m;
    float* v;
    long long n;
    float b1t, b2t;
};

static int newton_schulz(ns_model* m, float* X, int r, int c, int steps, float* out);
static size_t ns_scratch_floats(size_t mat, size_t gram);

// Optimizer update of all weights, or of those marked in `sel`.
static int optimizer_step(ns_model* m, float lr, const std::vector<char>* sel) {
    const Spec& s = m->spec;
    const std::string& mode = s.optimizer;
    const bool ref = mode == "reference";
    float b1, b2, eps, dec, omb1, omb2;
    if (ref) {
        b1 = 0.9f; b2 = 0.999f; eps = 1e-8f; dec = 0.01f; omb1 = 0.1f; omb2 = 0.001f;
    } else {
        double B1 = s.optv("beta1", 0.9), B2 = s.optv("beta2", 0.999);
        b1 = (float)B1; b2 = (float)B2;
        eps = (float)s.optv("eps", 1e-8);
        dec = (float)s.optv("decay", 0.01);
        omb1 = (float)(1.0 - B1);
        omb2 = (float)(1.0 - B2);
    }
    std::vector<AdamTensor> at;
    std::vector<char> fresh(s.weights.size(), 0);  // working copy written by the AdamW pass
    for (size_t wi = 0; wi < s.weights.size(); wi++) {
        if (sel && !(*sel)[wi]) {
            fresh[wi] = 1;  // not part of this update: leave its working copy alone
            continue;
        }
        const WeightInfo& w = s.weights[wi];
        const bool matrix = w.rows > 1 && w.cols > 1;
        const int mn = w.rows < w.cols ? w.rows : w.cols;
        float* W = m->d_w + w.off;
        float* G = m->d_g + w.off;
        if ((ref || mode == "muon") && matrix && mn >= 8) {
            const float mu = ref ? 0.95f : (float)s.optv("momentum", 0.95);
            const float mdec = ref ? 0.01f : (float)s.optv("decay", 0.01);
            launch_counter() += 1;
            muon_momentum(m->d_m + w.off, G, (long long)w.count, mu, m->stream);
            const float le = lr * sqrtf((float)mn);
            if (ref) {
                // reference: MGS in place on the momentum, then reset it
                launch_counter() += 2;
                mgs_orthonormalize(m->d_m + w.off, w.rows, w.cols, m->stream);
                muon_apply(W, m->d_m + w.off, m->d_m + w.off, (long long)w.count, le, mdec * lr, 1, m->stream);
            } else {
                if (newton_schulz(m, m->d_m + w.off, w.rows, w.cols, (int)s.optv("steps", 5), m->d_o)) return -1;
                // a flat bf16 working copy is written by the same pass
                const WkTarget wt = working_target(m, (int)wi);
                __nv_bfloat16* w16 = nullptr;
                if (wt.dst && wt.rows == 1 && m->wdt == kBF16) {
                    w16 = reinterpret_cast<__nv_bfloat16*>(wt.dst);
                    fresh[wi] = 1;
                }
                launch_counter() += 1;
                muon_apply(W, m->d_o, nullptr, (long long)w.count, le, mdec * lr, 0, m->stream, w16);
            }
        } else {
            long long t = ++m->adam_t[wi];
            AdamTensor a;
            a.w = W;
            a.g = G;
            a.m = m->d_m + w.off;
            a.v = m->d_v + w.off;
            a.n = (long long)w.count;
            a.b1t = 1.f - powf(b1, (float)t);
            a.b2t = 1.f - powf(b2, (float)t);
            const WkTarget wt = working_target(m, (int)wi);
            if (wt.dst) {
                a.wk = wt.dst;
                a.wk_ld = wt.ld;
                a.wk_cols = wt.cols;
                a.wk_off = wt.off;
                a.wk_bf16 = m->wdt == kBF16;
                fresh[wi] = 1;
            }
            at.push_back(a);
        }
    }
    if (!at.empty()) {
        AdamHyper h{lr, b1, b2, omb1, omb2, eps, dec};
        launch_counter() += (at.size() + kAdamBatch - 1) / kAdamBatch;
        if (adamw_multi(at.data(), (int)at.size(), h, m->stream)) return fail("adamw launch failed");
    }
    return refresh_working(m, &fresh);
}

// Scratch floats newton_schulz needs for a matrix of `mat` elements whose
// Gram matrix has `gram` elements (every sub-buffer 256-byte aligned).
static size_t ns_round(size_t x) { return (x + 63) & ~(size_t)63; }
static size_t ns_scratch_floats(size_t mat, size_t gram) {
    // fp32: Gram A, polynomial B, two iterates, norm partials;
    // bf16 operand copies: two iterates, A and B (half a float each)
    return 2 * ns_round(gram) + 2 * ns_round(mat) + 1024 + ns_round(mat) + ns_round(gram);
}

// X (r x c, fp32) -> out = NS5(X / ||X||), the quintic Newton-Schulz
// iteration Y' = a Y + (b A + c A^2) Y with A = Y Y^T (Y^T Y when r > c).
// Uses m->d_ns as scratch. In bf16 mode the three GEMMs of an iteration
// take bf16 operands (fp32 accumulation; the a Y and b A terms are added in
// fp32 from fp32 copies), as Muon's orthogonalisation is usually run;
// otherwise they run on fp32 operands (TF32 tensor cores, or the SIMT
// kernel in the fp32 parity mode).
static int newton_schulz(ns_model* m, float* X, int r, int c, int steps, float* out) {
    const bool tr = r > c;
    const int R = tr ? c : r;  // Gram size
    const size_t gram = ns_round((size_t)R * R), mat = ns_round((size_t)r * c);
    float* A = m->d_ns;
    float* B = A + gram;
    float* Y0 = B + gram;
    float* Y1 = Y0 + mat;
    float* part = Y1 + mat;
    const bool h = m->wdt == kBF16;
    __nv_bfloat16* Y0h = reinterpret_cast<__nv_bfloat16*>(part + 1024);
    __nv_bfloat16* Y1h = Y0h + mat;
    __nv_bfloat16* Ah = Y1h + mat;
    __nv_bfloat16* Bh = Ah + gram;
    const int dt = h ? kBF16 : kF32;
    launch_counter() += 2;
    if (frob_normalize(X, (long long)r * c, 1e-7f, Y0, part, m->stream, h ? Y0h : nullptr))
        return fail("normalisation launch failed");
    const float a = 3.4445f, b = -4.7750f, cc = 2.0315f;
    float* cur = Y0;
    float* nxt = Y1;
    __nv_bfloat16* curh = Y0h;
    __nv_bfloat16* nxth = Y1h;
    for (int it = 0; it < steps; it++) {
        const bool last = it + 1 == steps;
        const void* Yop = h ? (const void*)curh : (const void*)cur;
        GemmDesc g1;  // A = Y Y^T  (or Y^T Y)
        g1.M = R;
        g1.N = R;
        g1.K = tr ? r : c;
        g1.a = opnd(Yop, dt, c, tr);
        g1.b = opnd(Yop, dt, c, tr);
        g1.ep.c32 = A;
        g1.ep.ld_c32 = R;
        if (h) {
            g1.ep.c16 = Ah;
            g1.ep.ld_c16 = R;
        }
        if (run_gemm(m, g1)) return -1;
        GemmDesc g2;  // B = b A + c A A (A symmetric)
        g2.M = R;
        g2.N = R;
        g2.K = R;
        g2.a = opnd(h ? (const void*)Ah : (const void*)A, dt, R, false);
        g2.b = opnd(h ? (const void*)Ah : (const void*)A, dt, R, false);
        g2.ep.alpha = cc;
        g2.ep.add = A;
        g2.ep.ld_add = R;
        g2.ep.add_scale = b;
        if (h) {
            g2.ep.c16 = Bh;
            g2.ep.ld_c16 = R;
        } else {
            g2.ep.c32 = B;
            g2.ep.ld_c32 = R;
        }
        if (run_gemm(m, g2)) return -1;
        const void* Bop = h ? (const void*)Bh : (const void*)B;
        GemmDesc g3;  // Y' = a Y + B Y   (or a Y + Y B)
        g3.M = r;
        g3.N = c;
        if (!tr) {
            g3.K = R;
            g3.a = opnd(Bop, dt, R, false);
            g3.b = opnd(Yop, dt, c, true);
        } else {
            g3.K = R;
            g3.a = opnd(Yop, dt, c, false);
            g3.b = opnd(Bop, dt, R, false);
        }
        g3.ep.add = cur;
        g3.ep.ld_add = c;
        g3.ep.add_scale = a;
        g3.ep.c32 = last ? out : nxt;  // the last iterate goes straight to the output
        g3.ep.ld_c32 = c;
        if (h && !last) {
            g3.ep.c16 = nxth;
            g3.ep.ld_c16 = c;
        }
        if (run_gemm(m, g3)) return -1;
        std::swap(cur, nxt);
        std::swap(curh, nxth);
    }
    if (steps <= 0) cudaMemcpyAsync(out, cur, sizeof(float) * (size_t)r * c, cudaMemcpyDeviceToDevice, m->stream);
    return 0;
}

// ---------------------------------------------------------------------------
// synchronisation with error / timeout checks
// ---------------------------------------------------------------------------
// Wait (bounded by the model's timeout) until the communicator's last call
// has completed its enqueue; aborts the communicator on error or timeout.
static int nccl_settle(ns_model* m) {
    auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t st;
        nccl().CommGetAsyncError(m->comm, &st);
        if (st == ncclSuccess) {
            host_region_add(m, "host:nccl_enqueue",
                            std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count());
            return 0;
        }
        if (st != ncclInProgress) {
            nccl().CommAbort(m->comm);
            m->comm = nullptr;
            m->group_lost = true;
            return fail(std::string("NCCL error: ") + nccl().GetErrorString(st));
        }
        auto el = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
        if (el.count() > m->timeout_ms) {
            nccl().CommAbort(m->comm);
            m->comm = nullptr;
            m->group_lost = true;
            return fail("collective enqueue timed out");
        }
        std::this_thread::yield();
    }
}

static int finish(ns_model* m) {
    auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        cudaError_t q = cudaStreamQuery(m->stream);
        if (q == cudaSuccess) break;
        if (q != cudaErrorNotReady) return fail(std::string("CUDA error: ") + cudaGetErrorString(q));
        if (m->comm) {
            ncclResult_t ar;
            nccl().CommGetAsyncError(m->comm, &ar);
            if (ar != ncclSuccess && ar != ncclInProgress) {
                nccl().CommAbort(m->comm);
                m->comm = nullptr;
                m->group_lost = true;
                return fail(std::string("NCCL error: ") + nccl().GetErrorString(ar));
            }
            auto el = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
            if (el.count() > m->timeout_ms) {
                nccl().CommAbort(m->comm);
                m->comm = nullptr;
                m->group_lost = true;
                return fail("collective timed out");
            }
            // spin (yielding): a timed sleep oversleeps by tens of microseconds,
            // which would idle the GPU between steps
            std::this_thread::yield();
        } else {
            cudaError_t e = cudaStreamSynchronize(m->stream);
            if (e != cudaSuccess) return fail(std::string("CUDA error: ") + cudaGetErrorString(e));
            break;
        }
    }
    int herr = 0;
    cudaMemcpy(&herr, m->d_err, sizeof(int), cudaMemcpyDeviceToHost);
    if (herr) {
        cudaMemset(m->d_err, 0, sizeof(int));
        return fail("device pipeline wait timed out (code " + std::to_string(herr) + ")");
    }
    return 0;
}

static void sync_host(const ns_model* m) {
    if (!m->host_dirty) return;
    cudaMemcpy(m->h_w.data(), m->d_w, sizeof(float) * m->spec.total, cudaMemcpyDeviceToHost);
    m->host_dirty = false;
}

static int upload_weights(ns_model* m) {
    if (cudaMemcpy(m->d_w, m->h_w.data(), sizeof(float) * m->spec.total, cudaMemcpyHostToDevice) != cudaSuccess)
        return fail("weight upload failed");
    if (m->d_active && !m->moe_active.empty())
        cudaMemcpy(m->d_active, m->moe_active.data(), m->moe_active.size(), cudaMemcpyHostToDevice);
    if (refresh_working(m, nullptr)) return -1;
    return finish(m);
}

// ---------------------------------------------------------------------------
// public entry points
// ---------------------------------------------------------------------------
namespace {
struct SpecCache {
    std::mutex mu;
    std::map<std::string, std::unique_ptr<Spec>> specs;
};
SpecCache& spec_cache() {
    static SpecCache c;
    return c;
}
const Spec* cached_spec(const char* text) {
    if (!text) return nullptr;
    SpecCache& c = spec_cache();
    std::lock_guard<std::mutex> g(c.mu);
    auto it = c.specs.find(text);
    if (it != c.specs.end()) return it->second.get();
    std::unique_ptr<Spec> s(new Spec());
    std::string err;
    if (!parse_spec(text, *s, err)) {
        g_err = err;
        return nullptr;
    }
    const Spec* r = s.get();
    c.specs[text] = std::move(s);
    return r;
}
int env_precision(int def) {
    const char* e = getenv("NS_B200_PRECISION");
    if (!e) return def;
    std::string v(e);
    if (v == "fp32") return 0;
    if (v == "tf32") return 1;
    if (v == "bf16") return 2;
    return def;
}
}  // namespace

extern "C" {

const char* nsb_last_error(void) { return g_err.c_str(); }
const char* nsb_version(void) { return "ns-b200 0.1 (ABI " NS_RUNTIME_VERSION ")"; }

size_t nsb_spec_weight_count(const char* spec) {
    const Spec* s = cached_spec(spec);
    return s ? s->total : 0;
}

const ns_weight_layout* nsb_spec_layout(const char* spec) {
    const Spec* s = cached_spec(spec);
    return s ? &s->layout : nullptr;
}

static ns_model* init_one(const char* spec, const float* weights, size_t num_floats) {
    g_err.clear();
    if (!spec || !weights) {
        fail("null spec or weights");
        return nullptr;
    }
    ns_model* m = new ns_model();
    std::string err;
    if (!parse_spec(spec, m->spec, err)) {
        delete m;
        fail("spec: " + err);
        return nullptr;
    }
    if (num_floats != m->spec.total) {
        delete m;
        fail("weight count mismatch");
        return nullptr;
    }
    if (!build_graph(m, err)) {
        delete m;
        fail("spec: " + err);
        return nullptr;
    }
    m->precision = env_precision(m->spec.precision);
    m->timing = getenv("NS_B200_REGION_TIMING") != nullptr;
    m->wdt = m->precision == 2 ? kBF16 : kF32;
    cudaGetDevice(&m->device);
    bool ok = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) == cudaSuccess;
    ok = ok && cudaStreamCreateWithFlags(&m->wstream, cudaStreamNonBlocking) == cudaSuccess;
    ok = ok && cudaEventCreateWithFlags(&m->ev_ms, cudaEventDisableTiming) == cudaSuccess;
    ok = ok && cudaEventCreateWithFlags(&m->ev_sm, cudaEventDisableTiming) == cudaSuccess;
    ok = ok && cudaEventCreateWithFlags(&m->ev_emb, cudaEventDisableTiming) == cudaSuccess;
    const size_t n = m->spec.total;
    ok = ok && (m->d_err = (int*)persist_alloc(sizeof(int)));
    ok = ok && (m->d_w = (float*)persist_alloc(sizeof(float) * n));
    ok = ok && (m->d_g = (float*)persist_alloc(sizeof(float) * (n + 1)));
    ok = ok && (m->d_m = (float*)persist_alloc(sizeof(float) * n));
    ok = ok && (m->d_v = (float*)persist_alloc(sizeof(float) * n));
    ok = ok && cudaMallocHost(&m->h_loss, 16) == cudaSuccess;
    size_t maxmat = 0, maxgram = 0;
    for (auto& w : m->spec.weights) {
        if (w.count > maxmat) maxmat = w.count;
        size_t g = (size_t)(w.rows < w.cols ? w.rows : w.cols);
        if (g * g > maxgram) maxgram = g * g;
    }
    ok = ok && (m->d_o = (float*)persist_alloc(sizeof(float) * (maxmat + 1)));
    m->ns_floats = ns_scratch_floats(maxmat, maxgram);
    if (m->spec.optimizer == "muon") ok = ok && (m->d_ns = (float*)persist_alloc(sizeof(float) * m->ns_floats));
    m->adam_t.assign(m->spec.weights.size(), 0);
    m->h_w.assign(weights, weights + n);
    for (size_t li = 0; li < m->spec.layers.size(); li++)
        if (m->spec.layers[li].kind == "moe") {
            m->moe_layer = (int)li;
            int E = (int)m->spec.layers[li].geti("experts", 1);
            int K0 = (int)m->spec.layers[li].geti("initial", E);
            if (K0 <= 0 || K0 > E) K0 = E;
            m->moe_active.assign(E, 0);
            for (int e = 0; e < K0; e++) m->moe_active[e] = 1;
            m->moe_active_count = K0;
            ok = ok && (m->d_active = (uint8_t*)persist_alloc(E));
            break;
        }
    // column indices of index / scatter ops, int64 on the device
    for (auto& op : m->ops)
        if (ok && (op.kind == OP_INDEX || op.kind == OP_SCATTER)) {
            std::vector<int64_t> h(op.ints.begin(), op.ints.end());
            op.d_idx = (int64_t*)persist_alloc(sizeof(int64_t) * h.size());
            ok = op.d_idx && cudaMemcpy(op.d_idx, h.data(), sizeof(int64_t) * h.size(), cudaMemcpyHostToDevice) ==
                                 cudaSuccess;
        }
    ok = ok && alloc_working(m) == 0;
    if (!ok || upload_weights(m)) {
        std::string e = g_err.empty() ? "device allocation failed" : g_err;
        nsb_free(m);
        fail(e);
        return nullptr;
    }
    return m;
}

static void multi_detach(ns_model* m);
static int multi_attach(ns_model* m, const char* spec, const float* weights, size_t n, int gpus);

ns_model* nsb_runtime_init(const char* spec, const float* weights, size_t num_floats) {
    ns_model* m = init_one(spec, weights, num_floats);
    if (!m) return nullptr;
    // NS_B200_GPUS=N: this model also drives the next N-1 devices
    const char* e = getenv("NS_B200_GPUS");
    const int gpus = e ? atoi(e) : 1;
    if (gpus > 1 && multi_attach(m, spec, weights, num_floats, gpus)) {
        const std::string err = g_err;
        nsb_free(m);
        fail(err);
        return nullptr;
    }
    return m;
}

void nsb_free(ns_model* m) {
    if (!m) return;
    multi_detach(m);
    if (m->stream) cudaStreamSynchronize(m->stream);
    free_plan(m);
    free_working(m);
    for (void* p : {(void*)m->d_err, (void*)m->d_w, (void*)m->d_g, (void*)m->d_m, (void*)m->d_v, (void*)m->d_o,
                    (void*)m->d_ns, (void*)m->d_active})
        if (p) cudaFree(p);
    for (auto& op : m->ops)
        if (op.d_idx) cudaFree(op.d_idx);
    for (auto& r : m->regions) {
        for (auto& ev : r.pending) { cudaEventDestroy(ev.first); cudaEventDestroy(ev.second); }
        for (auto& ev : r.pool) { cudaEventDestroy(ev.first); cudaEventDestroy(ev.second); }
    }
    if (m->h_loss) cudaFreeHost(m->h_loss);
    if (m->h_targets) cudaFreeHost(m->h_targets);
    if (m->comm_stream) cudaStreamSynchronize(m->comm_stream);
    if (m->ev_in) cudaEventDestroy(m->ev_in);
    if (m->ev_out) cudaEventDestroy(m->ev_out);
    if (m->comm) nccl().CommDestroy(m->comm);
    for (cudaEvent_t e : m->dist_events) cudaEventDestroy(e);
    for (cudaEvent_t e : m->chunk_events) cudaEventDestroy(e);
    if (m->copy_stream) {
        cudaStreamSynchronize(m->copy_stream);
        cudaStreamDestroy(m->copy_stream);
    }
    if (m->comm_stream) cudaStreamDestroy(m->comm_stream);
    if (m->wstream) {
        cudaStreamSynchronize(m->wstream);
        cudaStreamDestroy(m->wstream);
    }
    if (m->ev_ms) cudaEventDestroy(m->ev_ms);
    if (m->ev_sm) cudaEventDestroy(m->ev_sm);
    if (m->ev_emb) cudaEventDestroy(m->ev_emb);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

size_t nsb_model_output_numel(const ns_model* m, size_t input_numel) {
    if (!m) return 0;
    return (input_numel / (size_t)m->spec.in_cols) * (size_t)m->spec.out_cols;
}

size_t nsb_model_weight_count(const ns_model* m) { return m ? m->spec.total : 0; }

int nsb_model_get_weights(const ns_model* m, float* out, size_t n) {
    if (!m || !out || n != m->spec.total) return -1;
    sync_host(m);
    memcpy(out, m->h_w.data(), n * sizeof(float));
    return 0;
}

static int for_replicas(ns_model* m, const std::function<int(ns_model*)>& fn);

int nsb_set_precision(ns_model* m, int mode) {
    if (!m || mode < 0 || mode > 2) return -1;
    if (!m->reps.empty() && for_replicas(m, [mode](ns_model* r) { return nsb_set_precision(r, mode); })) return -1;
    if (mode == m->precision) return 0;
    cudaStreamSynchronize(m->stream);
    free_plan(m);
    m->precision = mode;
    m->wdt = mode == 2 ? kBF16 : kF32;
    if (alloc_working(m) || refresh_working(m, nullptr)) return -1;
    return finish(m);
}

int nsb_get_precision(const ns_model* m) { return m ? m->precision : -1; }

long long nsb_last_launch_count(const ns_model* m) {
    if (!m) return 0;
    long long n = m->launches;
    for (const ns_model* r : m->reps) n += r->launches;
    return n;
}

int nsb_region_timing(ns_model* m, int enable) {
    if (!m) return -1;
    cudaStreamSynchronize(m->stream);
    regions_collect(m);
    for (auto& r : m->regions) {
        r.ms = 0;
        r.count = 0;
    }
    m->timing = enable != 0;
    return 0;
}

int nsb_region_count(ns_model* m) {
    if (!m) return 0;
    cudaStreamSynchronize(m->stream);
    regions_collect(m);
    return (int)m->regions.size();
}

int nsb_region_get(const ns_model* m, int i, const char** label, double* total_ms, long long* count) {
    if (!m || i < 0 || i >= (int)m->regions.size()) return -1;
    if (label) *label = m->regions[i].label.c_str();
    if (total_ms) *total_ms = m->regions[i].ms;
    if (count) *count = m->regions[i].count;
    return 0;
}

int nsb_model_get_gradients(const ns_model* m, float* out, size_t n) {
    if (!m || !out || n != m->spec.total) return -1;
    cudaStreamSynchronize(m->stream);
    return cudaMemcpy(out, m->d_g, n * sizeof(float), cudaMemcpyDeviceToHost) == cudaSuccess ? 0 : -1;
}

int nsb_model_get_input_gradient(const ns_model* m, float* out, size_t n) {
    if (!m || !out) return -1;
    if (!m->spec.input_grad) return fail("the spec has no 'grad input' statement");
    if (!m->reps.empty()) {
        // the rows of all replicas, in call order
        size_t total = (size_t)m->last_rows;
        for (const ns_model* r : m->reps) total += (size_t)r->last_rows;
        const size_t w = (size_t)m->spec.in_cols;
        if (n != total * w) return fail("size mismatch");
        size_t off = 0;
        for (int i = -1; i < (int)m->reps.size(); i++) {
            const ns_model* r = i < 0 ? m : m->reps[i];
            if (!r->last_rows) continue;
            if (!r->vals[0].gcur) return fail("no train step has formed an input gradient yet");
            cudaStreamSynchronize(r->stream);
            if (cudaMemcpy(out + off, r->vals[0].gcur, sizeof(float) * r->last_rows * w, cudaMemcpyDeviceToHost) !=
                cudaSuccess)
                return -1;
            off += (size_t)r->last_rows * w;
        }
        return 0;
    }
    const Val& x = m->vals[0];
    if (!m->last_rows || !x.gcur) return fail("no train step has formed an input gradient yet");
    if (n != (size_t)m->last_rows * m->spec.in_cols) return fail("size mismatch");
    cudaStreamSynchronize(m->stream);
    return cudaMemcpy(out, x.gcur, n * sizeof(float), cudaMemcpyDeviceToHost) == cudaSuccess ? 0 : -1;
}

static int rows_of(const ns_model* m, size_t input_numel) {
    return (int)(input_numel / (size_t)m->spec.in_cols);
}

int nsb_eval_infer_device(ns_model* m, const float* d_input, float* d_output, size_t input_numel, void* stream) {
    if (!m) return -1;
    g_err.clear();
    if (!m->reps.empty()) return fail("device-pointer entries take single-GPU models (NS_B200_GPUS unset)");
    const long long l0 = launch_counter();
    const int M = rows_of(m, input_numel);
    if (M <= 0) return 0;
    if (plan(m, M, false)) return -1;
    // the caller's stream (NULL = the legacy default stream); the engine runs
    // on its own stream, ordered after and before the caller's by events
    cudaStream_t us = stream ? (cudaStream_t)stream : cudaStreamLegacy;
    cudaEvent_t ev;
    if (us != m->stream) {
        cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
        cudaEventRecord(ev, us);
        cudaStreamWaitEvent(m->stream, ev, 0);
    }
    cudaMemcpyAsync(m->d_in, d_input, sizeof(float) * (size_t)M * m->spec.in_cols, cudaMemcpyDeviceToDevice,
                    m->stream);
    int rc = forward(m, M, false);
    if (!rc)
        cudaMemcpyAsync(d_output, m->vals[m->out_val].f32, sizeof(float) * (size_t)M * m->spec.out_cols,
                        cudaMemcpyDeviceToDevice, m->stream);
    if (us != m->stream) {
        cudaEventRecord(ev, m->stream);
        cudaStreamWaitEvent(us, ev, 0);
        cudaEventDestroy(ev);
    }
    m->launches = launch_counter() - l0;
    return rc;
}

// Rows per chunk of a pipelined host-buffer inference (0: one pass). Worth
// it when the output copy to page-locked host memory is large enough to
// dominate the call (8 MB and up): the rows are split into four chunks, in
// whole attention sequences (or 128-row tiles), and each chunk's output is
// copied back while the next chunk computes. Rows are independent, so the
// result is that of one pass up to the fp32 summation order of a GEMM that
// splits K at the smaller row count.
static int infer_chunk_rows(const ns_model* m, int M, const float* output) {
    const size_t out_bytes = (size_t)M * m->spec.out_cols * sizeof(float);
    if (out_bytes < (8u << 20)) return 0;
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, output) != cudaSuccess || at.type != cudaMemoryTypeHost) {
        cudaGetLastError();
        return 0;  // pageable destination: copies would block the host
    }
    int unit = 128;
    for (const auto& l : m->spec.layers)
        if (l.kind == "attention") {
            const int S = (int)l.geti("seq", 0);
            if (S <= 0) return 0;  // one sequence spans the call
            unit = S;
        }
    const int chunk = (M / 4 + unit - 1) / unit * unit;
    return chunk > 0 && chunk < M && M % unit == 0 ? chunk : 0;
}

static int eval_pipelined(ns_model* m, const float* input, float* output, int M, int chunk) {
    const Spec& s = m->spec;
    if (!m->copy_stream && cudaStreamCreateWithFlags(&m->copy_stream, cudaStreamNonBlocking) != cudaSuccess)
        return fail("stream creation failed");
    if (!m->d_stage && !(m->d_stage = (float*)plan_alloc(m, sizeof(float) * (size_t)m->mmax * s.out_cols)))
        return fail("device allocation failed");
    const int n = (M + chunk - 1) / chunk;
    while ((int)m->chunk_events.size() < n + 1) {
        cudaEvent_t e;
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return fail("event creation failed");
        m->chunk_events.push_back(e);
    }
    const float* out_dev = m->vals[m->out_val].f32;
    for (int c = 0; c < n; c++) {
        const int r0 = c * chunk, mc = M - r0 < chunk ? M - r0 : chunk;
        cudaMemcpyAsync(m->d_in, input + (size_t)r0 * s.in_cols, sizeof(float) * (size_t)mc * s.in_cols,
                        cudaMemcpyHostToDevice, m->stream);
        if (forward(m, mc, false)) return -1;
        float* st = m->d_stage + (size_t)r0 * s.out_cols;
        cudaMemcpyAsync(st, out_dev, sizeof(float) * (size_t)mc * s.out_cols, cudaMemcpyDeviceToDevice, m->stream);
        cudaEventRecord(m->chunk_events[c], m->stream);
        cudaStreamWaitEvent(m->copy_stream, m->chunk_events[c], 0);
        cudaMemcpyAsync(output + (size_t)r0 * s.out_cols, st, sizeof(float) * (size_t)mc * s.out_cols,
                        cudaMemcpyDeviceToHost, m->copy_stream);
    }
    // the engine stream (which finish() waits on) ends after the last copy
    cudaEventRecord(m->chunk_events[n], m->copy_stream);
    cudaStreamWaitEvent(m->stream, m->chunk_events[n], 0);
    return 0;
}

static int eval_infer_one(ns_model* m, const float* input, float* output, size_t input_numel) {
    if (!m) return -1;
    g_err.clear();
    const long long l0 = launch_counter();
    const int M = rows_of(m, input_numel);
    if (M <= 0) return 0;
    if (!input || !output) return fail("null input/output");
    if (plan(m, M, false)) return -1;
    if (const int chunk = infer_chunk_rows(m, M, output)) {
        if (eval_pipelined(m, input, output, M, chunk)) {
            finish(m);
            return -1;
        }
        m->launches = launch_counter() - l0;
        return finish(m);
    }
    cudaMemcpyAsync(m->d_in, input, sizeof(float) * (size_t)M * m->spec.in_cols, cudaMemcpyHostToDevice, m->stream);
    if (forward(m, M, false)) {
        finish(m);
        return -1;
    }
    cudaMemcpyAsync(output, m->vals[m->out_val].f32, sizeof(float) * (size_t)M * m->spec.out_cols,
                    cudaMemcpyDeviceToHost, m->stream);
    m->launches = launch_counter() - l0;
    return finish(m);
}

static int train_core(ns_model* m, int M, const float* d_labels, const int* d_targets, float* loss_out, float lr,
                      bool train) {
    m->ce_fused = train && d_targets && !d_labels && m->d_tlogit && ce_fusable_producer(m);
    m->ce_targets = d_targets;
    if (forward(m, M, train)) return -1;
    int rl = region_begin(m, m->ce_fused ? "loss.fused" : "loss");
    if (loss_and_seed(m, M, d_labels, d_targets, train)) return -1;
    region_end(m, rl);
    launch_counter() += 1;
    const float scale = 1.0f / ((float)M * (m->spec.loss == "mse" ? (float)m->spec.out_cols : 1.f));
    if (train) {
        for (auto& v : m->vals) v.gcur = nullptr;
        Val& o = m->vals[m->out_val];
        o.gcur = o.gbuf;
        if (m->world > 1 && !m->comm) return fail("data-parallel group lost (an earlier collective failed)");
        // the loss sum rides at the end of the gradient blob (reduced with the last range)
        launch_counter() += 1;
        reduce_sum(m->d_rowloss, M, 1.0f, m->d_g + m->spec.total, m->stream);
        if (dist_active(m)) {
            m->reduced.assign(m->spec.weights.size(), 0);
            m->ev_next = 0;
            m->bucket_w.clear();
            m->bucket_done.clear();
            m->bucket_evt.clear();
        }
        if (backward(m, M)) return -1;
        if (dist_active(m)) {
            if (dist_reduce_finish(m) || dist_optimizer(m, lr)) return -1;
        } else {
            int ro = region_begin(m, "optimizer");
            if (optimizer_step(m, lr)) return -1;
            region_end(m, ro);
        }
        m->host_dirty = true;
        const float gscale = 1.0f / ((float)M * (float)m->world *
                                     (m->spec.loss == "mse" ? (float)m->spec.out_cols : 1.f));
        launch_counter() += 1;
        reduce_sum(m->d_g + m->spec.total, 1, gscale, m->d_loss, m->stream);
    } else {
        reduce_sum(m->d_rowloss, M, scale, m->d_loss, m->stream);
    }
    if (loss_out) cudaMemcpyAsync(m->h_loss, m->d_loss, sizeof(float), cudaMemcpyDeviceToHost, m->stream);
    return 0;
}

// ---------------------------------------------------------------------------
// One-hot labels read on the host. ns_runtime_train_step / ns_objective_loss
// take dense fp32 labels [M, C]; for the cross-entropy of the reference
// (loss = sum over y > 0 of -log p, seed = (p - y) / denom) a row holding a
// single 1.0 and zeros elsewhere is exactly the class index t, and an all-zero
// row is an index outside [0, C) (loss 0, seed p / denom). Host threads read
// the labels once; when every row is of these two kinds only the M indices
// cross PCIe (64 KB instead of 537 MB for c4) and the step takes the
// integer-target path. Any other row (smoothed or soft labels, a single
// value other than 1.0) keeps the dense copy and the dense loss kernel.
// ---------------------------------------------------------------------------
namespace {
struct ScanPool {
    std::vector<std::thread> th;
    std::mutex mu, job_mu;
    std::condition_variable cv, done_cv;
    std::function<void(int, int)> fn;  // (worker, workers)
    long long gen = 0;
    int pending = 0, n = 0;
    ScanPool() {
        // one worker per hardware thread up to 64; NS_B200_SCAN_THREADS overrides
        const unsigned hc = std::thread::hardware_concurrency();
        n = hc == 0 ? 4 : (int)(hc < 64u ? hc : 64u);
        if (const char* e = getenv("NS_B200_SCAN_THREADS")) {
            const int v = atoi(e);
            if (v > 0 && v <= 256) n = v;
        }
        for (int i = 0; i < n; i++) th.emplace_back([this, i] { loop(i); });
    }
    void loop(int i) {
        long long seen = 0;
        for (;;) {
            std::function<void(int, int)> f;
            {
                std::unique_lock<std::mutex> l(mu);
                cv.wait(l, [&] { return gen != seen; });
                seen = gen;
                f = fn;
            }
            f(i, n);
            std::lock_guard<std::mutex> l(mu);
            if (--pending == 0) done_cv.notify_all();
        }
    }
    // runs f on every worker and returns when all are done (one job at a time)
    void run(std::function<void(int, int)> f) {
        std::lock_guard<std::mutex> jl(job_mu);
        std::unique_lock<std::mutex> l(mu);
        fn = std::move(f);
        pending = n;
        gen++;
        cv.notify_all();
        done_cv.wait(l, [&] { return pending == 0; });
    }
};
// Created on first use and never destroyed: its threads wait on a condition
// variable until the process exits.
ScanPool& scan_pool() {
    static ScanPool* p = new ScanPool();
    return *p;
}

// The class of a one-hot row: its column, -1 for an all-zero row, -2 for any
// other row. Zero is tested on the magnitude bits (-0.0 counts as zero); the
// row is streamed 64 bytes at a time (eight 64-bit words OR-ed together), and
// only a block with a nonzero value is looked at element by element.
int onehot_col(const float* x, int C) {
    const uint32_t* u = reinterpret_cast<const uint32_t*>(x);
    int col = -1;
    auto one = [&](int k) -> bool {
        const uint32_t b = u[k];
        if ((b & 0x7fffffffu) == 0) return true;
        if (b != 0x3f800000u || col >= 0) return false;  // not 1.0f, or a second nonzero
        col = k;
        return true;
    };
    int c = 0;
    // unaligned head up to an 8-byte boundary
    while (c < C && (reinterpret_cast<uintptr_t>(u + c) & 7))
        if (!one(c++)) return -2;
    const uint64_t kMag = 0x7fffffff7fffffffull;
    for (; c + 16 <= C; c += 16) {
        const uint64_t* w = reinterpret_cast<const uint64_t*>(u + c);
        const uint64_t o = ((w[0] | w[1]) | (w[2] | w[3])) | ((w[4] | w[5]) | (w[6] | w[7]));
        if (!(o & kMag)) continue;
        for (int k = 0; k < 16; k++)
            if (!one(c + k)) return -2;
    }
    for (; c < C; c++)
        if (!one(c)) return -2;
    return col;
}
}  // namespace

// Reads M label rows into m->h_targets; true when every row is one-hot or
// all-zero.
static bool labels_as_targets(ns_model* m, const float* labels, int M) {
    const char* e = getenv("NS_B200_LABEL_SCAN");
    if ((e && e[0] == '0') || m->spec.loss == "mse") return false;
    const int C = m->spec.out_cols;
    if (C < 16) return false;  // small rows: the dense copy costs nothing
    if (m->h_targets_cap < M) {
        if (m->h_targets) cudaFreeHost(m->h_targets);
        m->h_targets = nullptr;
        m->h_targets_cap = 0;
        if (cudaMallocHost(&m->h_targets, sizeof(int) * (size_t)M) != cudaSuccess) {
            cudaGetLastError();
            m->h_targets = nullptr;
            return false;
        }
        m->h_targets_cap = M;
    }
    int* tg = m->h_targets;
    std::atomic<int> dense{0};
    scan_pool().run([&](int w, int nw) {
        const int r0 = (int)((long long)M * w / nw), r1 = (int)((long long)M * (w + 1) / nw);
        for (int r = r0; r < r1 && !dense.load(std::memory_order_relaxed); r++) {
            const int t = onehot_col(labels + (size_t)r * C, C);
            if (t == -2) {
                dense.store(1, std::memory_order_relaxed);
                return;
            }
            tg[r] = t;
        }
    });
    return dense.load() == 0;
}

static int train_entry(ns_model* m, const float* input, const float* labels, const int* targets, size_t input_numel,
                       float* loss_out, float lr, bool train, bool device_ptrs, void* stream) {
    if (!m) return -1;
    g_err.clear();
    const long long l0 = launch_counter();
    const int M = rows_of(m, input_numel);
    if (M <= 0) return fail("empty batch");
    if (!input || (!labels && !targets)) return fail("null input/labels");
    if (plan(m, M, true)) return -1;
    cudaMemcpyKind k = device_ptrs ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    cudaStream_t us = stream ? (cudaStream_t)stream : cudaStreamLegacy;
    if (device_ptrs) {
        // inputs are produced on the caller's stream: order after it on the GPU
        if (!m->ev_in && cudaEventCreateWithFlags(&m->ev_in, cudaEventDisableTiming) != cudaSuccess)
            return fail("event creation failed");
        cudaEventRecord(m->ev_in, us);
        cudaStreamWaitEvent(m->stream, m->ev_in, 0);
    }
    cudaMemcpyAsync(m->d_in, input, sizeof(float) * (size_t)M * m->spec.in_cols, k, m->stream);
    const float* dl = nullptr;
    const int* dt = nullptr;
    if (labels && !device_ptrs && labels_as_targets(m, labels, M)) {
        // every label row is one-hot (or all zero): send the class indices
        cudaMemcpyAsync(m->d_targets, m->h_targets, sizeof(int) * (size_t)M, cudaMemcpyHostToDevice, m->stream);
        dt = m->d_targets;
    } else if (labels) {
        cudaMemcpyAsync(m->d_labels, labels, sizeof(float) * (size_t)M * m->spec.out_cols, k, m->stream);
        dl = m->d_labels;
    } else {
        cudaMemcpyAsync(m->d_targets, targets, sizeof(int) * (size_t)M, k, m->stream);
        dt = m->d_targets;
    }
    float lr_eff = lr;
    if (train) {
        long long st = m->lr_step;
        if (st < 9223372036854775807LL) m->lr_step = st + 1;
        lr_eff = lr * lr_schedule(m, st);
    }
    const auto h0 = std::chrono::steady_clock::now();
    int rc = train_core(m, M, dl, dt, loss_out, lr_eff, train);
    if (train) {
        m->drop_step++;  // the next step draws fresh dropout masks
        m->last_rows = M;
    }
    m->launches = launch_counter() - l0;
    const auto h1 = std::chrono::steady_clock::now();
    if (device_ptrs && !loss_out && !rc) {
        // stream-ordered: later work on the caller's stream follows this step;
        // device errors surface at the next synchronising call
        if (!m->ev_out && cudaEventCreateWithFlags(&m->ev_out, cudaEventDisableTiming) != cudaSuccess)
            return fail("event creation failed");
        cudaEventRecord(m->ev_out, m->stream);
        cudaStreamWaitEvent(us, m->ev_out, 0);
        host_region_add(m, "host:launch", std::chrono::duration<double, std::milli>(h1 - h0).count());
        return cudaGetLastError() == cudaSuccess ? 0 : fail("kernel launch failed");
    }
    int rf = finish(m);
    host_region_add(m, "host:launch", std::chrono::duration<double, std::milli>(h1 - h0).count());
    host_region_add(m, "host:wait",
                    std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - h1).count());
    if (rc || rf) return -1;
    if (loss_out) *loss_out = *m->h_loss;
    return 0;
}

static int multi_train(ns_model* m, const float* input, const float* labels, const int* targets, size_t input_numel,
                       float* loss_out, float lr, bool train);
static int multi_infer(ns_model* m, const float* input, float* output, size_t input_numel);

int nsb_eval_infer(ns_model* m, const float* input, float* output, size_t input_numel) {
    if (m && !m->reps.empty()) return multi_infer(m, input, output, input_numel);
    return eval_infer_one(m, input, output, input_numel);
}

int nsb_runtime_train_step(ns_model* m, const float* input, const float* labels, size_t input_numel, float* loss_out,
                           float lr) {
    if (m && !m->reps.empty()) return multi_train(m, input, labels, nullptr, input_numel, loss_out, lr, true);
    return train_entry(m, input, labels, nullptr, input_numel, loss_out, lr, true, false, nullptr);
}

int nsb_runtime_train_step_idx(ns_model* m, const float* input, const int* targets, size_t input_numel,
                               float* loss_out, float lr) {
    if (m && !m->reps.empty()) return multi_train(m, input, nullptr, targets, input_numel, loss_out, lr, true);
    return train_entry(m, input, nullptr, targets, input_numel, loss_out, lr, true, false, nullptr);
}

int nsb_train_step_device(ns_model* m, const float* d_input, const float* d_labels, const int* d_targets,
                          size_t input_numel, float* loss_out, float lr, void* stream) {
    if (m && !m->reps.empty()) return fail("device-pointer entries take single-GPU models (NS_B200_GPUS unset)");
    return train_entry(m, d_input, d_labels, d_targets, input_numel, loss_out, lr, true, true, stream);
}

int nsb_objective_loss(ns_model* m, const float* input, const float* labels, size_t input_numel, float* loss_out) {
    if (m && !m->reps.empty()) return multi_train(m, input, labels, nullptr, input_numel, loss_out, 0.f, false);
    return train_entry(m, input, labels, nullptr, input_numel, loss_out, 0.f, false, false, nullptr);
}

// ---- checkpoints (reference codegen.cpp:2501-2557) --------------------------
int nsb_save_checkpoint(const ns_model* m, const char* path) {
    if (!m || !path) return -1;
    sync_host(m);
    FILE* fp = fopen(path, "wb");
    if (!fp) return -1;
    const unsigned magic = 0x4E534D32u;
    const size_t n = m->spec.total;
    bool ok = fwrite(&magic, sizeof(magic), 1, fp) == 1 && fwrite(&n, sizeof(n), 1, fp) == 1 &&
              fwrite(m->h_w.data(), sizeof(float), n, fp) == n;
    if (ok && m->moe_layer >= 0) {
        const unsigned nl = 1u;
        const size_t cap = m->moe_active.size();
        ok = fwrite(&nl, sizeof(nl), 1, fp) == 1 && fwrite(&cap, sizeof(cap), 1, fp) == 1 &&
             fwrite(m->moe_active.data(), 1, cap, fp) == cap;
    }
    fclose(fp);
    return ok ? 0 : -1;
}

int nsb_load_checkpoint(ns_model* m, const char* path) {
    if (!m || !path) return -1;
    if (!m->reps.empty() && for_replicas(m, [path](ns_model* r) { return nsb_load_checkpoint(r, path); })) return -1;
    FILE* fp = fopen(path, "rb");
    if (!fp) return -1;
    unsigned magic = 0;
    size_t n = 0;
    std::vector<float> w(m->spec.total);
    bool ok = fread(&magic, sizeof(magic), 1, fp) == 1 && fread(&n, sizeof(n), 1, fp) == 1 &&
              (magic == 0x4E534D31u || magic == 0x4E534D32u) && n == m->spec.total &&
              fread(w.data(), sizeof(float), n, fp) == n;
    std::vector<uint8_t> mask = m->moe_active;
    if (ok && m->moe_layer >= 0) {
        if (magic == 0x4E534D32u) {
            unsigned nl = 0;
            size_t cap = 0;
            ok = fread(&nl, sizeof(nl), 1, fp) == 1 && fread(&cap, sizeof(cap), 1, fp) == 1 && nl == 1u &&
                 cap == mask.size() && fread(mask.data(), 1, cap, fp) == cap;
        } else {
            mask.assign(mask.size(), 1);
        }
    }
    fclose(fp);
    if (!ok) return -1;
    cudaStreamSynchronize(m->stream);
    m->h_w = w;
    m->host_dirty = false;
    if (m->moe_layer >= 0) {
        m->moe_active = mask;
        m->moe_active_count = 0;
        for (uint8_t a : mask) m->moe_active_count += a;
    }
    return upload_weights(m) ? -1 : 0;
}

// ---- MoE expert lifecycle (reference CPU emit, codegen.cpp:2559-2625) -------
struct MoeGeom {
    size_t cap, dim, ffn, off_g, off_e1, off_e2;
    bool linear;
};
static bool moe_geom(const ns_model* m, MoeGeom& g) {
    if (m->moe_layer < 0) return false;
    const LayerSpec& l = m->spec.layers[m->moe_layer];
    g.cap = (size_t)l.geti("experts", 1);
    g.dim = (size_t)l.geti("dim", 1);
    g.linear = l.gets("expert", "ffn") == "linear";
    g.ffn = g.linear ? g.dim : (size_t)l.geti("ffn", 4 * (long long)g.dim);
    for (auto& w : m->spec.weights) {
        if (w.layer != m->moe_layer) continue;
        if (w.name == l.name + "_g_w") g.off_g = w.off;
        else if (w.name == l.name + "_e1_w") g.off_e1 = w.off;
        else if (w.name == l.name + "_e2_w") g.off_e2 = w.off;
    }
    return true;
}

size_t nsb_expert_count(const ns_model* m) { return m ? m->moe_active_count : 0; }

size_t nsb_expert_kill(ns_model* m, int k) {
    if (!m || m->moe_layer < 0) return m ? m->moe_active_count : 0;
    if (!m->reps.empty()) for_replicas(m, [k](ns_model* r) { nsb_expert_kill(r, k); return 0; });
    if (k < 0 || k >= (int)m->moe_active.size() || !m->moe_active[k]) return m->moe_active_count;
    m->moe_active[k] = 0;
    m->moe_active_count--;
    cudaMemcpy(m->d_active, m->moe_active.data(), m->moe_active.size(), cudaMemcpyHostToDevice);
    return m->moe_active_count;
}

// Re-pack the working copies of the MoE layer's expert weights after the
// master blob changed on the device (the host mirror is stale from then on).
static int moe_weights_changed(ns_model* m) {
    std::vector<char> done(m->spec.weights.size(), 1);
    for (size_t w = 0; w < m->spec.weights.size(); w++)
        if (m->spec.weights[w].layer == m->moe_layer) done[w] = 0;
    m->host_dirty = true;
    if (refresh_working(m, &done)) return -1;
    return finish(m);
}

static nsb::ExpertGeom expert_geom(const MoeGeom& g) {
    nsb::ExpertGeom e;
    e.cap = g.cap;
    e.dim = g.dim;
    e.n1 = g.dim * g.ffn;
    e.off_g = g.off_g;
    e.off_e1 = g.off_e1;
    e.off_e2 = g.off_e2;
    e.linear = g.linear;
    return e;
}

size_t nsb_expert_merge(ns_model* m, int a, int b) {
    MoeGeom g;
    if (!m || !moe_geom(m, g)) return m ? m->moe_active_count : 0;
    if (!m->reps.empty()) for_replicas(m, [a, b](ns_model* r) { nsb_expert_merge(r, a, b); return 0; });
    const int cap = (int)g.cap;
    if (a < 0 || b < 0 || a == b || a >= cap || b >= cap || !m->moe_active[a] || !m->moe_active[b])
        return m->moe_active_count;
    // on the device blob: expert a := (a + b) / 2, then b leaves the mask
    launch_counter() += 1;
    if (expert_merge_device(m->d_w, expert_geom(g), a, b, m->stream)) return m->moe_active_count;
    m->moe_active[b] = 0;
    m->moe_active_count--;
    cudaMemcpyAsync(m->d_active, m->moe_active.data(), m->moe_active.size(), cudaMemcpyHostToDevice, m->stream);
    moe_weights_changed(m);
    return m->moe_active_count;
}

size_t nsb_expert_birth(ns_model* m, int n) {
    MoeGeom g;
    if (!m || !moe_geom(m, g) || n <= 0) return m ? m->moe_active_count : 0;
    // every replica draws the same sources and noise (same generator state)
    if (!m->reps.empty()) for_replicas(m, [n](ns_model* r) { nsb_expert_birth(r, n); return 0; });
    if (m->moe_active_count >= g.cap) return m->moe_active_count;
    // the source and the noise come from the model's generator in the CPU
    // runtime's order (gate column, e1, e2 per new expert); only the noise
    // travels to the device, where the new expert is written
    int src = (int)(m->rng() % g.cap);
    size_t tries = 0;
    while (tries++ < g.cap && !m->moe_active[src]) src = (int)(m->rng() % g.cap);
    const size_t n1 = g.dim * g.ffn;
    const size_t per = g.dim + n1 * (g.linear ? 1 : 2);
    std::vector<float> noise(per);
    float* d_noise = nullptr;
    if (cudaMalloc(&d_noise, per * sizeof(float)) != cudaSuccess) {
        fail("device allocation failed");
        return m->moe_active_count;
    }
    const nsb::ExpertGeom eg = expert_geom(g);
    for (int e = 0; e < (int)g.cap && n > 0; e++) {
        if (m->moe_active[e]) continue;
        for (size_t i = 0; i < per; i++) noise[i] = ((float)(m->rng() % 1001) / 1000.f - 0.5f) * 1e-2f;
        cudaMemcpyAsync(d_noise, noise.data(), per * sizeof(float), cudaMemcpyHostToDevice, m->stream);
        launch_counter() += 1;
        expert_birth_device(m->d_w, eg, src, e, d_noise, m->stream);
        cudaStreamSynchronize(m->stream);  // the host noise buffer is reused by the next expert
        m->moe_active[e] = 1;
        m->moe_active_count++;
        n--;
    }
    cudaFree(d_noise);
    cudaMemcpyAsync(m->d_active, m->moe_active.data(), m->moe_active.size(), cudaMemcpyHostToDevice, m->stream);
    moe_weights_changed(m);
    return m->moe_active_count;
}

// ---- data parallel ----------------------------------------------------------
}  // extern "C"

// Muon matrices are sharded over the ranks: matrix k (in weight order) is
// updated by rank k % world only. NS_B200_SHARD_MUON=0 keeps every update
// replicated.
static bool takes_muon(const ns_model* m, const WeightInfo& w) {
    const std::string& mode = m->spec.optimizer;
    const int mn = w.rows < w.cols ? w.rows : w.cols;
    return (mode == "reference" || mode == "muon") && w.rows > 1 && w.cols > 1 && mn >= 8;
}

void assign_owners(ns_model* m) {
    const char* e = getenv("NS_B200_SHARD_MUON");
    const bool on = !(e && e[0] == '0');
    m->owner.assign(m->spec.weights.size(), -1);
    if (!on || m->world <= 1) return;
    int k = 0;
    for (size_t w = 0; w < m->spec.weights.size(); w++)
        if (takes_muon(m, m->spec.weights[w])) m->owner[w] = k++ % m->world;
}

extern "C" {

int nsb_dist_unique_id(void* id128) {
    if (!id128) return -1;
    if (!nccl().ok) return fail("libnccl.so.2 not loadable");
    ncclUniqueId id;
    if (nccl().GetUniqueId(&id) != ncclSuccess) return fail("ncclGetUniqueId failed");
    memcpy(id128, &id, sizeof(id));
    return 0;
}

static int dist_init_one(ns_model* m, int rank, int world, const void* id128, int timeout_ms);

int nsb_dist_init(ns_model* m, int rank, int world, const void* id128, int timeout_ms) {
    if (!m || !id128 || world < 1 || rank < 0 || rank >= world) return -1;
    if (!m->reps.empty()) return fail("a model driving several GPUs in-call cannot also join a process group");
    return dist_init_one(m, rank, world, id128, timeout_ms);
}

}  // extern "C"

static int dist_init_one(ns_model* m, int rank, int world, const void* id128, int timeout_ms) {
    m->timeout_ms = timeout_ms > 0 ? timeout_ms : 60000;
    if (world == 1) {
        m->world = 1;
        m->rank = 0;
        return 0;
    }
    if (!nccl().ok) return fail("libnccl.so.2 not loadable");
    ncclUniqueId id;
    memcpy(&id, id128, sizeof(id));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    // The all-reduces run beside the backward GEMMs: cap the SMs NCCL may
    // occupy (NS_B200_NCCL_MAX_CTAS, default 16, measured best on two GPUs
    // against 8 and NCCL's own choice; 0 leaves the choice to NCCL).
    {
        const char* e = getenv("NS_B200_NCCL_MAX_CTAS");
        const int mx = e ? atoi(e) : 16;
        if (mx > 0) {
            cfg.maxCTAs = mx;
            cfg.minCTAs = 1;
        }
    }
    ncclComm_t comm = nullptr;
    ncclResult_t r = nccl().CommInitRankConfig(&comm, world, id, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) return fail(std::string("nccl init: ") + nccl().GetErrorString(r));
    auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t st;
        nccl().CommGetAsyncError(comm, &st);
        if (st == ncclSuccess) break;
        if (st != ncclInProgress) {
            nccl().CommAbort(comm);
            return fail(std::string("nccl init: ") + nccl().GetErrorString(st));
        }
        auto el = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
        if (el.count() > m->timeout_ms) {
            nccl().CommAbort(comm);
            return fail("nccl init timed out");
        }
        std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
    if (!m->comm_stream && cudaStreamCreateWithFlags(&m->comm_stream, cudaStreamNonBlocking) != cudaSuccess) {
        nccl().CommAbort(comm);
        return fail("communication stream creation failed");
    }
    m->comm = comm;
    m->rank = rank;
    m->world = world;
    assign_owners(m);
    return 0;
}

// ---------------------------------------------------------------------------
// In-call multi-GPU: the reference host calls ns_runtime_train_step /
// ns_eval_infer once with the whole batch; with NS_B200_GPUS=N set at
// ns_runtime_init the model holds N-1 replicas on the next devices, joined
// with it by NCCL (the data-parallel path above: gradients all-reduced,
// Muon matrices sharded). Each call splits the caller's rows (in whole
// attention sequences) over the N models, which run at the same time, the
// lead on the calling thread and each replica on a worker thread of its own;
// each copies its slice of the host buffers straight in and out.
// ---------------------------------------------------------------------------
namespace nsb {

struct ReplicaWorker {
    std::thread th;
    std::mutex mu;
    std::condition_variable cv;
    std::function<int()> job;
    bool has_job = false, done = false, quit = false;
    int rc = 0;
    std::string err;
    int device = 0;

    void loop() {
        cudaSetDevice(device);
        for (;;) {
            std::function<int()> j;
            {
                std::unique_lock<std::mutex> lk(mu);
                cv.wait(lk, [&] { return has_job || quit; });
                if (!has_job) return;
                j = std::move(job);
                has_job = false;
            }
            g_err.clear();
            const int r = j();
            std::lock_guard<std::mutex> g(mu);
            rc = r;
            err = g_err;
            done = true;
            cv.notify_all();
        }
    }
    void post(std::function<int()> f) {
        std::lock_guard<std::mutex> g(mu);
        job = std::move(f);
        has_job = true;
        done = false;
        cv.notify_all();
    }
    int wait(std::string& e) {
        std::unique_lock<std::mutex> lk(mu);
        cv.wait(lk, [&] { return done; });
        e = err;
        return rc;
    }
};

struct ReplicaPool {
    std::vector<std::unique_ptr<ReplicaWorker>> w;
};

}  // namespace nsb

// fn(model, index) on the lead (index 0, calling thread, lead device
// current) and on every replica (its worker thread) at the same time.
static int run_all(ns_model* m, const std::function<int(ns_model*, int)>& fn) {
    const size_t n = m->reps.size();
    for (size_t i = 0; i < n; i++) {
        ns_model* r = m->reps[i];
        m->pool->w[i]->post([&fn, r, i] { return fn(r, (int)i + 1); });
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(m->device);
    int rc = fn(m, 0);
    std::string err = rc ? g_err : std::string();
    for (size_t i = 0; i < n; i++) {
        std::string e;
        if (m->pool->w[i]->wait(e) && !rc) {
            rc = -1;
            err = "GPU " + std::to_string(m->reps[i]->device) + ": " + e;
        }
    }
    cudaSetDevice(prev);
    if (rc) return fail(err);
    return 0;
}

// fn on every replica (not the lead), each on its worker thread.
static int for_replicas(ns_model* m, const std::function<int(ns_model*)>& fn) {
    return run_all(m, [&fn](ns_model* r, int i) { return i == 0 ? 0 : fn(r); });
}

static int multi_attach(ns_model* m, const char* spec, const float* weights, size_t n, int gpus) {
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || gpus > count)
        return fail("NS_B200_GPUS=" + std::to_string(gpus) + " but " + std::to_string(count) + " GPUs are visible");
    if (!nccl().ok) return fail("libnccl.so.2 not loadable");
    for (const auto& l : m->spec.layers)
        if (l.kind == "attention" && l.geti("seq", 0) <= 0)
            return fail("NS_B200_GPUS: attention over the whole call (seq 0) cannot be split across GPUs");
    int prev = 0;
    cudaGetDevice(&prev);
    m->pool = new nsb::ReplicaPool();
    for (int i = 1; i < gpus; i++) {
        const int dev = (m->device + i) % count;
        cudaSetDevice(dev);
        ns_model* r = init_one(spec, weights, n);
        if (!r) {
            cudaSetDevice(prev);
            return -1;
        }
        nsb_set_precision(r, m->precision);
        m->reps.push_back(r);
        auto w = std::unique_ptr<nsb::ReplicaWorker>(new nsb::ReplicaWorker());
        w->device = dev;
        nsb::ReplicaWorker* wp = w.get();
        w->th = std::thread([wp] { wp->loop(); });
        m->pool->w.push_back(std::move(w));
    }
    cudaSetDevice(prev);
    // one communicator per device, all ranks joining at once
    ncclUniqueId id;
    if (nccl().GetUniqueId(&id) != ncclSuccess) return fail("ncclGetUniqueId failed");
    const int timeout = 60000;
    return run_all(m, [&id, gpus, timeout](ns_model* r, int rank) {
        return dist_init_one(r, rank, gpus, &id, timeout);
    });
}

static void multi_detach(ns_model* m) {
    if (!m->pool) return;
    for (auto& w : m->pool->w) {
        {
            std::lock_guard<std::mutex> g(w->mu);
            w->quit = true;
            w->cv.notify_all();
        }
        if (w->th.joinable()) w->th.join();
    }
    int prev = 0;
    cudaGetDevice(&prev);
    for (ns_model* r : m->reps) {
        cudaSetDevice(r->device);
        nsb_free(r);
    }
    cudaSetDevice(prev);
    m->reps.clear();
    delete m->pool;
    m->pool = nullptr;
}

// Rows of one indivisible unit: an attention sequence, else a row.
static int split_unit(const ns_model* m) {
    int unit = 1;
    for (const auto& l : m->spec.layers)
        if (l.kind == "attention") unit = (int)l.geti("seq", 1);
    return unit > 0 ? unit : 1;
}

// [row0, rows) per model: whole units, as even as possible, in call order.
static std::vector<std::pair<int, int>> split_rows(const ns_model* m, int M) {
    const int parts = 1 + (int)m->reps.size(), unit = split_unit(m);
    const int units = M / unit, base = units / parts, extra = units % parts;
    std::vector<std::pair<int, int>> out;
    int r0 = 0;
    for (int i = 0; i < parts; i++) {
        int rows = (base + (i < extra ? 1 : 0)) * unit;
        if (i == parts - 1) rows = M - r0;  // a ragged tail (not whole units) stays with the last
        out.push_back(std::make_pair(r0, rows));
        r0 += rows;
    }
    return out;
}

static int multi_infer(ns_model* m, const float* input, float* output, size_t input_numel) {
    g_err.clear();
    const int M = rows_of(m, input_numel);
    if (M <= 0) return 0;
    if (!input || !output) return fail("null input/output");
    const auto parts = split_rows(m, M);
    const int in_cols = m->spec.in_cols, out_cols = m->spec.out_cols;
    return run_all(m, [&](ns_model* r, int i) {
        const int r0 = parts[i].first, rows = parts[i].second;
        if (rows <= 0) return 0;
        return eval_infer_one(r, input + (size_t)r0 * in_cols, output + (size_t)r0 * out_cols,
                              (size_t)rows * in_cols);
    });
}

static int multi_train(ns_model* m, const float* input, const float* labels, const int* targets, size_t input_numel,
                       float* loss_out, float lr, bool train) {
    g_err.clear();
    const int M = rows_of(m, input_numel);
    const int parts_n = 1 + (int)m->reps.size(), unit = split_unit(m);
    if (M <= 0) return fail("empty batch");
    if (!input || (!labels && !targets)) return fail("null input/labels");
    if (train && M % (parts_n * unit) != 0)
        return fail("NS_B200_GPUS: a train step's rows must split evenly over the GPUs in whole sequences (" +
                    std::to_string(M) + " rows, " + std::to_string(parts_n) + " GPUs, unit " + std::to_string(unit) +
                    ")");
    const auto parts = split_rows(m, M);
    const int in_cols = m->spec.in_cols, out_cols = m->spec.out_cols;
    std::vector<float> losses(parts_n, 0.f);
    const int rc = run_all(m, [&](ns_model* r, int i) {
        const int r0 = parts[i].first, rows = parts[i].second;
        if (rows <= 0) return 0;  // inference-only objective: nothing to do
        return train_entry(r, input + (size_t)r0 * in_cols, labels ? labels + (size_t)r0 * out_cols : nullptr,
                           targets ? targets + r0 : nullptr, (size_t)rows * in_cols, loss_out ? &losses[i] : nullptr,
                           lr, train, false, nullptr);
    });
    if (rc) return -1;
    if (loss_out) {
        if (train) {
            *loss_out = losses[0];  // the loss sum rode the all-reduce: every rank holds the global mean
        } else {
            double s = 0.0;  // per-model means over their rows, weighted by rows
            for (int i = 0; i < parts_n; i++) s += (double)losses[i] * parts[i].second;
            *loss_out = (float)(s / M);
        }
    }
    return 0;
}