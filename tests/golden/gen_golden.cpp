// Golden-vector generator for the oracle pins (test infrastructure).
//
// Part 1 (kernel level): this file #includes one CPU translation unit that
// the reference compiler emitted (`nsc model.ns --cpp --runtime`; every such
// unit carries every static helper) and calls the helpers directly, the way
// the reference's own tests/test_transformer.cpp:97-98 does.
// Part 2 (ABI level): dlopen()s reference-emitted runtime libraries
// (oracle/_ref/libref_*.so) and drives them through ns_runtime.h.
//
// Inputs come from the shared generator (oracle/nsrand.h via orc_fill_*,
// compiled without FP contraction in oracle/nsrand.c). Every array is
// written as a .npy file into the output directory given as argv[1].
//
// Build/run: tests/golden/gen_golden.py.
#include REF_TU

#include <dlfcn.h>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

extern "C" {
void orc_fill_uniform(float* out, size_t n, uint64_t seed, double lo, double hi);
void orc_fill_normal(float* out, size_t n, uint64_t seed, double mu, double sd);
void orc_fill_tokens(float* out, size_t n, uint64_t seed, int64_t vocab);
}

static std::string g_dir;

static void save_npy(const std::string& name, const void* data, const char* descr, size_t elem,
                     std::vector<size_t> shape) {
    std::string hdr = "{'descr': '" + std::string(descr) + "', 'fortran_order': False, 'shape': (";
    size_t n = 1;
    for (size_t i = 0; i < shape.size(); i++) {
        hdr += std::to_string(shape[i]);
        if (shape.size() == 1 || i + 1 < shape.size()) hdr += ",";
        if (i + 1 < shape.size()) hdr += " ";
        n *= shape[i];
    }
    hdr += "), }";
    size_t total = 10 + hdr.size() + 1;
    size_t pad = (64 - total % 64) % 64;
    hdr += std::string(pad, ' ');
    hdr += "\n";
    std::string path = g_dir + "/" + name + ".npy";
    FILE* f = fopen(path.c_str(), "wb");
    if (!f) { perror(path.c_str()); exit(1); }
    const unsigned char magic[8] = {0x93, 'N', 'U', 'M', 'P', 'Y', 1, 0};
    fwrite(magic, 1, 8, f);
    unsigned short hl = (unsigned short)hdr.size();
    fwrite(&hl, 2, 1, f);
    fwrite(hdr.data(), 1, hdr.size(), f);
    fwrite(data, elem, n, f);
    fclose(f);
}
static void savef(const std::string& name, const std::vector<float>& v, std::vector<size_t> shape) {
    save_npy(name, v.data(), "<f4", 4, shape);
}
static void saved(const std::string& name, const std::vector<double>& v, std::vector<size_t> shape) {
    save_npy(name, v.data(), "<f8", 8, shape);
}
static std::vector<float> U(size_t n, uint64_t seed, double lo, double hi) {
    std::vector<float> v(n); orc_fill_uniform(v.data(), n, seed, lo, hi); return v;
}
static std::vector<float> N(size_t n, uint64_t seed, double mu, double sd) {
    std::vector<float> v(n); orc_fill_normal(v.data(), n, seed, mu, sd); return v;
}
static std::vector<double> row_sums(const std::vector<float>& v, size_t rows, size_t cols) {
    std::vector<double> s(rows, 0.0);
    for (size_t r = 0; r < rows; r++)
        for (size_t c = 0; c < cols; c++) s[r] += (double)v[r * cols + c];
    return s;
}

static void kernels() {
    {   // dense forward + both gradients
        const int64_t M = 37, K = 29, Nn = 23;
        auto A = U(M * K, 101, -1, 1), B = U(K * Nn, 102, -1, 1), dC = U(M * Nn, 103, -1, 1);
        std::vector<float> C(M * Nn), dA(M * K), dB(K * Nn);
        ns_matmul(A.data(), B.data(), C.data(), M, K, Nn);
        ns_matmul_grad_a(dC.data(), B.data(), dA.data(), M, K, Nn);
        ns_matmul_grad_w(A.data(), dC.data(), dB.data(), M, K, Nn);
        savef("matmul_C", C, {37, 23}); savef("matmul_dA", dA, {37, 29}); savef("matmul_dB", dB, {29, 23});
    }
    {   // activations and derivatives, codes 0..6
        const size_t n = 2000;
        auto x = U(n, 110, -6, 6);
        std::vector<float> a(7 * n), d(7 * n);
        for (int c = 0; c < 7; c++)
            for (size_t i = 0; i < n; i++) { a[c * n + i] = ns_act2(x[i], c); d[c * n + i] = ns_act_deriv(x[i], c); }
        savef("act_y", a, {7, n}); savef("act_dy", d, {7, n});
    }
    {   // layernorm forward / backward
        const int64_t R = 13, L = 48;
        auto x = N(R * L, 120, 0.3, 2.0), dout = N(R * L, 121, 0, 1);
        std::vector<float> y = x, dx(R * L);
        ns_layernorm(y.data(), y.size(), L);
        ns_layernorm_grad(dout.data(), x.data(), dx.data(), dx.size(), L);
        savef("ln_y", y, {13, 48}); savef("ln_dx", dx, {13, 48});
    }
    {   // softmax
        auto x = N(60, 190, 0, 3);
        ns_softmax(x.data(), 60, 10);
        savef("softmax_y", x, {6, 10});
    }
    {   // embedding gather / scatter-add with out-of-range and fractional ids
        const int64_t V = 11, D = 8;
        std::vector<float> idx = {0, 3, 10, -1, 11, 3.7f, 2.2f, 5, 5, 0, -0.5f, 7};
        auto W = N(V * D, 130, 0, 1), dout = N(idx.size() * D, 131, 0, 1);
        std::vector<float> out(idx.size() * D), dW(V * D);
        ns_embedding(W.data(), idx.data(), out.data(), (int64_t)idx.size(), V, D);
        ns_embedding_grad_w(dout.data(), idx.data(), dW.data(), idx.size(), D, V);
        savef("emb_out", out, {idx.size(), 8}); savef("emb_dW", dW, {11, 8});
    }
    struct AttnCase { const char* tag; int64_t B, S, D, H; uint64_t seed; };
    const AttnCase acs[] = {{"attn_a", 3, 8, 16, 4, 140}, {"attn_b", 2, 64, 64, 2, 240}};
    for (const auto& c : acs) {   // attention forward / backward, per-sequence S
        const int64_t BS = c.B * c.S, D = c.D;
        auto x = N(BS * D, c.seed, 0, 1);
        auto Wq = N(D * D, c.seed + 1, 0, 0.25), Wk = N(D * D, c.seed + 2, 0, 0.25);
        auto Wv = N(D * D, c.seed + 3, 0, 0.25), Wo = N(D * D, c.seed + 4, 0, 0.25);
        auto dout = N(BS * D, c.seed + 5, 0, 1);
        std::vector<float> q(BS * D), k(BS * D), v(BS * D), sc(c.S * c.S), proj(BS * D), out(BS * D);
        ns_attention_fwd(x.data(), Wq.data(), Wk.data(), Wv.data(), Wo.data(), q.data(), k.data(),
                         v.data(), sc.data(), proj.data(), out.data(), BS, D, c.H, c.S);
        std::vector<float> dX(BS * D), dWq(D * D), dWk(D * D), dWv(D * D), dWo(D * D);
        ns_attention_bwd(dout.data(), x.data(), Wq.data(), Wk.data(), Wv.data(), Wo.data(),
                         dX.data(), nullptr, nullptr, nullptr, nullptr, BS, D, c.H, c.S);
        ns_attention_bwd(dout.data(), x.data(), Wq.data(), Wk.data(), Wv.data(), Wo.data(),
                         nullptr, dWq.data(), nullptr, nullptr, nullptr, BS, D, c.H, c.S);
        ns_attention_bwd(dout.data(), x.data(), Wq.data(), Wk.data(), Wv.data(), Wo.data(),
                         nullptr, nullptr, dWk.data(), nullptr, nullptr, BS, D, c.H, c.S);
        ns_attention_bwd(dout.data(), x.data(), Wq.data(), Wk.data(), Wv.data(), Wo.data(),
                         nullptr, nullptr, nullptr, dWv.data(), nullptr, BS, D, c.H, c.S);
        ns_attention_bwd(dout.data(), x.data(), Wq.data(), Wk.data(), Wv.data(), Wo.data(),
                         nullptr, nullptr, nullptr, nullptr, dWo.data(), BS, D, c.H, c.S);
        std::string t = c.tag;
        size_t bs = (size_t)BS, d = (size_t)D;
        savef(t + "_out", out, {bs, d}); savef(t + "_dX", dX, {bs, d});
        savef(t + "_dWq", dWq, {d, d}); savef(t + "_dWk", dWk, {d, d});
        savef(t + "_dWv", dWv, {d, d}); savef(t + "_dWo", dWo, {d, d});
    }
    {   // MoE forward and the four gradients, with one dead expert
        const int64_t M = 37, D = 8, E = 4, H = 16;
        const uint8_t active[4] = {1, 1, 0, 1};
        auto x = N(M * D, 150, 0, 1), Wg = N(D * E, 151, 0, 0.5);
        auto We1 = N(E * D * H, 152, 0, 0.35), We2 = N(E * H * D, 153, 0, 0.35), dout = N(M * D, 154, 0, 1);
        std::vector<float> out(M * D), dx(M * D, 0.f), dWg(D * E), dWe1(E * D * H), dWe2(E * H * D);
        ns_moe_fwd(x.data(), Wg.data(), We1.data(), We2.data(), active, out.data(), M, D, H, E);
        ns_moe_grad_x(dout.data(), x.data(), Wg.data(), We1.data(), We2.data(), active, dx.data(), M, D, H, E);
        ns_moe_grad_wg(dout.data(), x.data(), Wg.data(), We1.data(), We2.data(), active, dWg.data(), M, D, H, E);
        ns_moe_grad_we1(dout.data(), x.data(), Wg.data(), We1.data(), We2.data(), active, dWe1.data(), M, D, H, E);
        ns_moe_grad_we2(dout.data(), x.data(), Wg.data(), We1.data(), We2.data(), active, dWe2.data(), M, D, H, E);
        savef("moe_out", out, {37, 8}); savef("moe_dx", dx, {37, 8}); savef("moe_dWg", dWg, {8, 4});
        savef("moe_dWe1", dWe1, {4, 128}); savef("moe_dWe2", dWe2, {4, 128});
    }
    {   // routing at the config-3 router scale (D=1024, E=8): each expert's
        // output differs, so row sums pin the top-1 decision of every token.
        const int64_t M = 1024, D = 1024, E = 8, H = 8;
        auto x = N(M * D, 160, 0, 1), Wg = N(D * E, 161, 0, 0.02);
        auto We1 = N(E * D * H, 162, 0, 1.0 / 32), We2 = N(E * H * D, 163, 0, 1.0 / 32);
        std::vector<float> out(M * D);
        ns_moe_fwd(x.data(), Wg.data(), We1.data(), We2.data(), nullptr, out.data(), M, D, H, E);
        saved("route_rowsum", row_sums(out, M, D), {1024});
    }
    {   // cross-entropy seed and loss
        const int64_t R = 9, C = 7;
        auto p = N(R * C, 170, 0, 2);
        std::vector<float> y(R * C, 0.f), d(R * C);
        for (int64_t r = 0; r < R; r++) y[r * C + (r * 3) % C] = 1.f;
        ns_loss_grad(p.data(), y.data(), d.data(), d.size(), C);
        std::vector<float> l = {ns_cross_entropy(p.data(), y.data(), p.size(), C)};
        savef("ce_d", d, {9, 7}); savef("ce_loss", l, {1});
    }
    {   // modified Gram-Schmidt, both orientations
        auto G = N(12 * 9, 180, 0, 1), G2 = N(5 * 11, 181, 0, 1);
        ns_orthonom(G.data(), 12, 9); ns_orthonom(G2.data(), 5, 11);
        savef("mgs_a", G, {12, 9}); savef("mgs_b", G2, {5, 11});
    }
    {   // elementwise binops (all four codes, full-size right operand)
        auto A = U(7 * 13, 190, -2, 2), B = U(7 * 13, 191, 0.5, 2);
        for (int code = 0; code < 4; code++) {
            std::vector<float> C(7 * 13);
            ns_binop(A.data(), A.size(), B.data(), B.size(), C.data(), code);
            savef("binop_" + std::to_string(code), C, {7, 13});
        }
        savef("binop_a", A, {7, 13}); savef("binop_b", B, {7, 13});
    }
    {   // data movement: the reference's CPU helpers on a [9, 11] tensor; the
        // scatters repeat an index so the write order is pinned
        const int64_t R = 9, C = 11;
        auto X = U(R * C, 195, -1, 1), Y = U(R * 5, 196, -1, 1), Z = U(4 * C, 197, -1, 1);
        std::vector<float> t(R * C), c2(R * (C + 5)), c0((R + 4) * C), s2(R * 6), sr(3 * C), i2(R * 4), ir(3 * C),
            sc(R * C), scr(R * C);
        const int64_t idx_c[4] = {7, 2, 7, 0};   // columns (7 repeated)
        const int64_t idx_r[3] = {5, 1, 5};      // rows (5 repeated)
        const int64_t upd_c[5] = {3, 9, 3, 1, 10};
        const int64_t upd_r[4] = {2, 6, 2, 8};
        ns_transpose2d(X.data(), t.data(), R, C);
        ns_concat2(X.data(), Y.data(), c2.data(), R, C, 5);
        ns_concat0(X.data(), Z.data(), c0.data(), R, 4, C);
        ns_slice2(X.data(), s2.data(), R, C, 3, 9);
        ns_slicerows(X.data(), sr.data(), C, 2, 5);
        ns_index2(X.data(), idx_c, i2.data(), R, C, 4);
        ns_indexrows(X.data(), idx_r, ir.data(), 3, C);
        ns_scatter2(X.data(), upd_c, Y.data(), sc.data(), R, C, 5);
        ns_scatterrows(X.data(), upd_r, Z.data(), scr.data(), R, C, 4);
        savef("dm_x", X, {(size_t)R, (size_t)C}); savef("dm_y", Y, {(size_t)R, 5}); savef("dm_z", Z, {4, (size_t)C});
        savef("dm_transpose", t, {(size_t)C, (size_t)R});
        savef("dm_concat2", c2, {(size_t)R, (size_t)C + 5});
        savef("dm_concat0", c0, {(size_t)R + 4, (size_t)C});
        savef("dm_slice2", s2, {(size_t)R, 6});
        savef("dm_slicerows", sr, {3, (size_t)C});
        savef("dm_index2", i2, {(size_t)R, 4});
        savef("dm_indexrows", ir, {3, (size_t)C});
        savef("dm_scatter2", sc, {(size_t)R, (size_t)C});
        savef("dm_scatterrows", scr, {(size_t)R, (size_t)C});
    }
}

// ---- ABI level -------------------------------------------------------------
struct RefLib {
    void* h;
    template <class F> F sym(const char* n) {
        void* p = dlsym(h, n);
        if (!p) { fprintf(stderr, "missing %s\n", n); exit(1); }
        return (F)p;
    }
};
static RefLib load(const std::string& name) {
    std::string p = std::string(REF_DIR) + "/libref_" + name + ".so";
    void* h = dlopen(p.c_str(), RTLD_NOW | RTLD_LOCAL);
    if (!h) { fprintf(stderr, "%s\n", dlerror()); exit(1); }
    return RefLib{h};
}
typedef void* (*init_t)(const float*, size_t);
typedef int (*infer_t)(void*, const float*, float*, size_t);
typedef int (*train_t)(void*, const float*, const float*, size_t, float*, float);
typedef int (*obj_t)(void*, const float*, const float*, size_t, float*);
typedef int (*getw_t)(const void*, float*, size_t);
typedef size_t (*wcount_t)(void);
typedef int (*ckpt_t)(const void*, const char*);
typedef size_t (*ecount_t)(const void*);
typedef size_t (*ebirth_t)(void*, int);
typedef size_t (*emerge_t)(void*, int, int);
typedef size_t (*ekill_t)(void*, int);

static std::vector<float> file_bytes_as_u8(const std::string& path) {
    FILE* f = fopen(path.c_str(), "rb");
    std::vector<float> out;
    int c;
    while ((c = fgetc(f)) != EOF) out.push_back((float)c);
    fclose(f);
    return out;
}

// Weights: layer l of the blob is N(0, sd_l) from seed base + l.
static std::vector<float> make_blob(const std::vector<size_t>& counts, const std::vector<double>& sds, uint64_t base) {
    std::vector<float> w;
    for (size_t l = 0; l < counts.size(); l++) {
        auto p = N(counts[l], base + l, 0, sds[l]);
        w.insert(w.end(), p.begin(), p.end());
    }
    return w;
}

static void train_case(const char* tag, const std::vector<size_t>& counts, const std::vector<double>& sds,
                       uint64_t wseed, const std::vector<float>& x, size_t in_numel, int classes,
                       uint64_t lseed, int steps, float lr, bool moe) {
    RefLib L = load(tag);
    auto init = L.sym<init_t>("ns_runtime_init");
    auto train = L.sym<train_t>("ns_runtime_train_step");
    auto obj = L.sym<obj_t>("ns_objective_loss");
    auto getw = L.sym<getw_t>("ns_model_get_weights");
    auto infer = L.sym<infer_t>("ns_eval_infer");
    auto save = L.sym<ckpt_t>("ns_save_checkpoint");
    auto w = make_blob(counts, sds, wseed);
    size_t rows = x.size() / in_numel;
    std::vector<float> tgt(rows);
    orc_fill_tokens(tgt.data(), rows, lseed, classes);
    std::vector<float> y(rows * classes, 0.f);
    for (size_t r = 0; r < rows; r++) y[r * classes + (size_t)tgt[r]] = 1.f;
    void* m = init(w.data(), w.size());
    if (!m) { fprintf(stderr, "%s: weight count mismatch\n", tag); exit(1); }
    std::vector<float> losses(steps);
    for (int s = 0; s < steps; s++) train(m, x.data(), y.data(), x.size(), &losses[s], lr);
    std::vector<float> wout(w.size());
    getw(m, wout.data(), wout.size());
    float ol = 0.f;
    obj(m, x.data(), y.data(), x.size(), &ol);
    std::vector<float> out(rows * classes);
    infer(m, x.data(), out.data(), x.size());
    std::string t = tag;
    savef(t + "_w0", w, {w.size()}); savef(t + "_x", x, {x.size()}); savef(t + "_y", y, {rows, (size_t)classes});
    savef(t + "_losses", losses, {(size_t)steps}); savef(t + "_w", wout, {wout.size()});
    savef(t + "_obj", std::vector<float>{ol}, {1}); savef(t + "_out", out, {rows, (size_t)classes});
    std::string ck = g_dir + "/" + t + ".ckpt";
    save(m, ck.c_str());
    auto bytes = file_bytes_as_u8(ck);
    remove(ck.c_str());
    savef(t + "_ckpt_bytes", bytes, {bytes.size()});
    if (moe) {
        auto count = L.sym<ecount_t>("ns_expert_count");
        auto kill = L.sym<ekill_t>("ns_expert_kill");
        auto merge = L.sym<emerge_t>("ns_expert_merge");
        std::vector<float> counts_seen;
        counts_seen.push_back((float)count(m));
        counts_seen.push_back((float)kill(m, 1));
        counts_seen.push_back((float)kill(m, 1));       // already dead: unchanged
        counts_seen.push_back((float)merge(m, 0, 2));
        counts_seen.push_back((float)merge(m, 0, 0));   // invalid: unchanged
        std::vector<float> wl(w.size());
        getw(m, wl.data(), wl.size());
        infer(m, x.data(), out.data(), x.size());
        savef(t + "_lifecycle_counts", counts_seen, {counts_seen.size()});
        savef(t + "_lifecycle_w", wl, {wl.size()});
        savef(t + "_lifecycle_out", out, {rows, (size_t)classes});
        save(m, ck.c_str());
        auto b2 = file_bytes_as_u8(ck);
        remove(ck.c_str());
        savef(t + "_lifecycle_ckpt_bytes", b2, {b2.size()});
        // birth into the two dead slots: a random live source plus noise,
        // both from the runtime's generator
        auto birth = L.sym<ebirth_t>("ns_expert_birth");
        std::vector<float> bc{(float)birth(m, 2)};
        std::vector<float> wb(w.size());
        getw(m, wb.data(), wb.size());
        infer(m, x.data(), out.data(), x.size());
        savef(t + "_birth_count", bc, {1});
        savef(t + "_birth_w", wb, {wb.size()});
        savef(t + "_birth_out", out, {rows, (size_t)classes});
    }
}

static void abi() {
    {   // config 1 forward, 64 rows
        RefLib L = load("c1");
        auto init = L.sym<init_t>("ns_runtime_init");
        auto infer = L.sym<infer_t>("ns_eval_infer");
        auto w = make_blob({784 * 1024, 1024 * 1024, 1024 * 10},
                           {1 / 28.0, 1 / 32.0, 1 / 32.0}, 211);
        auto x = U(64 * 784, 201, -1, 1);
        void* m = init(w.data(), w.size());
        std::vector<float> out(64 * 10);
        infer(m, x.data(), out.data(), x.size());
        savef("c1_out", out, {64, 10});
    }
    {   // config 2 forward, two 256-token sequences, one call per sequence
        RefLib L = load("c2");
        auto init = L.sym<init_t>("ns_runtime_init");
        auto infer = L.sym<infer_t>("ns_eval_infer");
        auto w = make_blob({8192 * 512, 512 * 512, 512 * 512, 512 * 512, 512 * 512, 512 * 2048, 2048 * 512},
                           {0.02, 0.02, 0.02, 0.02, 0.02, 0.02, 0.02}, 311);
        std::vector<float> tok(512);
        orc_fill_tokens(tok.data(), 512, 301, 8192);
        void* m = init(w.data(), w.size());
        std::vector<float> out(512 * 512);
        infer(m, tok.data(), out.data(), 256);
        infer(m, tok.data() + 256, out.data() + 256 * 512, 256);
        saved("c2_rowsum", row_sums(out, 512, 512), {512});
        // rows 0..127 of each sequence (256 rows)
        std::vector<float> rows(out.begin(), out.begin() + 128 * 512);
        rows.insert(rows.end(), out.begin() + 256 * 512, out.begin() + 384 * 512);
        savef("c2_rows", rows, {256, 512});
    }
    {   // config 3 forward (FFN experts), 64 tokens
        RefLib L = load("c3");
        auto init = L.sym<init_t>("ns_runtime_init");
        auto infer = L.sym<infer_t>("ns_eval_infer");
        auto w = make_blob({1024 * 8, 8 * 1024 * 1024, 8 * 1024 * 1024}, {0.02, 1 / 32.0, 1 / 32.0}, 411);
        auto x = N(64 * 1024, 401, 0, 1);
        void* m = init(w.data(), w.size());
        std::vector<float> out(64 * 1024);
        infer(m, x.data(), out.data(), x.size());
        saved("c3_rowsum", row_sums(out, 64, 1024), {64});
        savef("c3_rows", out, {64, 1024});
    }
    // small training runs through ns_runtime_train_step (reference optimizer)
    train_case("tmlp", {6 * 16, 16 * 8, 8 * 4}, {0.41, 0.25, 0.35}, 501, U(16 * 6, 502, -1, 1), 6, 4,
               503, 40, 0.05f, false);
    {
        std::vector<float> tok(64);
        orc_fill_tokens(tok.data(), 64, 602, 32);
        train_case("ttfm", {32 * 6, 6 * 6, 6 * 6, 6 * 6, 6 * 6, 6 * 12, 12 * 6, 6 * 16},
                   {0.5, 0.4, 0.4, 0.4, 0.4, 0.4, 0.3, 0.4}, 601, tok, 1, 16, 603, 30, 0.01f, false);
    }
    {
        std::vector<float> tok(24);
        orc_fill_tokens(tok.data(), 24, 702, 16);
        train_case("tmoe", {16 * 8, 8 * 4, 4 * 8 * 16, 4 * 16 * 8, 8 * 4},
                   {0.5, 0.5, 0.35, 0.25, 0.35}, 701, tok, 1, 4, 703, 30, 0.01f, true);
    }
}

int main(int argc, char** argv) {
    if (argc < 2) { fprintf(stderr, "usage: %s outdir\n", argv[0]); return 2; }
    g_dir = argv[1];
    kernels();
    abi();
    return 0;
}
