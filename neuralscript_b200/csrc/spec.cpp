// Spec parser (host only). Mirrors neuralscript_b200/spec.py.
#include "spec.h"

#include <algorithm>
#include <sstream>

namespace nsb {

int act_code(const std::string& n0) {
    std::string n = n0;
    std::transform(n.begin(), n.end(), n.begin(), ::tolower);
    if (n == "identity" || n == "none" || n == "linear") return 0;
    if (n == "relu") return 1;
    if (n == "leaky_relu" || n == "leakyrelu") return 2;
    if (n == "sigmoid") return 3;
    if (n == "tanh") return 4;
    if (n == "silu" || n == "swish") return 5;
    if (n == "gelu") return 6;
    return -1;
}

int data_fn_values(const std::string& fn) {
    if (fn == "concat") return 2;
    if (fn == "slice") return 1;
    if (fn == "index") return 1;
    if (fn == "scatter") return 2;
    return -1;
}

static std::string trim(const std::string& s) {
    size_t a = s.find_first_not_of(" \t\r\n");
    if (a == std::string::npos) return "";
    size_t b = s.find_last_not_of(" \t\r\n");
    return s.substr(a, b - a + 1);
}

static std::vector<std::string> split_ws(const std::string& s) {
    std::istringstream is(s);
    std::vector<std::string> out;
    std::string t;
    while (is >> t) out.push_back(t);
    return out;
}

static bool kv(const std::vector<std::string>& tok, size_t from, std::map<std::string, std::string>& out,
               std::string& err) {
    for (size_t i = from; i < tok.size(); i++) {
        size_t e = tok[i].find('=');
        if (e == std::string::npos) {
            err = "expected key=value, got '" + tok[i] + "'";
            return false;
        }
        out[tok[i].substr(0, e)] = tok[i].substr(e + 1);
    }
    return true;
}

bool parse_spec(const std::string& text, Spec& s, std::string& err) {
    s = Spec();
    s.text = text;
    std::istringstream in(text);
    std::string raw;
    int lineno = 0;
    try {
        while (std::getline(in, raw)) {
            lineno++;
            std::string line = raw.substr(0, raw.find('#'));
            line = trim(line);
            if (line.empty()) continue;
            auto tok = split_ws(line);
            bool assign = tok.size() > 1 && (tok[1] == "=" || tok[0].find('=') != std::string::npos);
            if (assign && tok[0] != "layer" && tok[0] != "optimizer" && tok[0] != "schedule") {
                size_t e = line.find('=');
                std::string lhs = trim(line.substr(0, e)), rhs = trim(line.substr(e + 1));
                size_t lp = rhs.find('('), rp = rhs.rfind(')');
                if (lp == std::string::npos || rp == std::string::npos || rp < lp) {
                    err = "line " + std::to_string(lineno) + ": expected v = f(args)";
                    return false;
                }
                SpecOp op;
                op.out = lhs;
                op.fn = trim(rhs.substr(0, lp));
                std::string args = rhs.substr(lp + 1, rp - lp - 1);
                std::istringstream as(args);
                std::string a;
                while (std::getline(as, a, ',')) {
                    a = trim(a);
                    if (!a.empty()) op.args.push_back(a);
                }
                const int nv = data_fn_values(op.fn);
                if (nv >= 0) {
                    // value operands first, then integers
                    if ((int)op.args.size() < nv) { err = "line " + std::to_string(lineno) + ": " + op.fn + " needs " + std::to_string(nv) + " values"; return false; }
                    for (size_t i = nv; i < op.args.size(); i++) {
                        size_t used = 0;
                        long long v = std::stoll(op.args[i], &used);
                        if (used != op.args[i].size()) { err = "line " + std::to_string(lineno) + ": expected an integer, got '" + op.args[i] + "'"; return false; }
                        op.ints.push_back(v);
                    }
                    op.args.resize(nv);
                }
                s.ops.push_back(op);
                continue;
            }
            const std::string& kw = tok[0];
            if (kw == "network") {
                if (tok.size() > 1) s.name = tok[1];
            } else if (kw == "input") {
                if (tok.size() < 2) { err = "input needs a width or 'tokens'"; return false; }
                if (tok[1] == "tokens") {
                    s.tokens = true;
                    s.in_cols = 1;
                } else {
                    s.in_cols = std::stoi(tok[1]);
                }
            } else if (kw == "layer") {
                if (tok.size() < 3) { err = "line " + std::to_string(lineno) + ": layer <name> <kind> ..."; return false; }
                LayerSpec l;
                l.name = tok[1];
                l.kind = tok[2];
                std::transform(l.kind.begin(), l.kind.end(), l.kind.begin(), ::tolower);
                if (!kv(tok, 3, l.p, err)) return false;
                s.layers.push_back(l);
            } else if (kw == "output") {
                if (tok.size() > 1) s.output = tok[1];
            } else if (kw == "loss") {
                if (tok.size() > 1) s.loss = tok[1];
            } else if (kw == "optimizer") {
                if (tok.size() > 1) s.optimizer = tok[1];
                std::map<std::string, std::string> m;
                if (!kv(tok, 2, m, err)) return false;
                for (auto& e : m) s.opt[e.first] = std::stod(e.second);
            } else if (kw == "schedule") {
                if (tok.size() > 1) s.schedule = tok[1];
                std::map<std::string, std::string> m;
                if (!kv(tok, 2, m, err)) return false;
                for (auto& e : m) s.sched[e.first] = std::stod(e.second);
            } else if (kw == "grad") {
                if (tok.size() != 2 || tok[1] != "input") { err = "line " + std::to_string(lineno) + ": expected 'grad input'"; return false; }
                s.input_grad = true;
            } else if (kw == "precision") {
                if (tok.size() > 1) {
                    if (tok[1] == "fp32") s.precision = 0;
                    else if (tok[1] == "tf32") s.precision = 1;
                    else if (tok[1] == "bf16") s.precision = 2;
                    else { err = "unknown precision " + tok[1]; return false; }
                }
            } else {
                err = "line " + std::to_string(lineno) + ": unknown statement '" + kw + "'";
                return false;
            }
        }
    } catch (const std::exception& e) {
        err = std::string("bad number in spec: ") + e.what();
        return false;
    }
    if (s.ops.empty()) { err = "spec has no operations"; return false; }
    if (s.input_grad && s.tokens) { err = "grad input needs a real-valued input (token ids have no gradient)"; return false; }
    if (s.output.empty()) s.output = s.ops.back().out;

    // weights in layer-declaration order
    size_t off = 0;
    for (size_t li = 0; li < s.layers.size(); li++) {
        const LayerSpec& l = s.layers[li];
        auto add = [&](const std::string& n, long long r, long long c) {
            WeightInfo w;
            w.name = n;
            w.rows = (int)r;
            w.cols = (int)c;
            w.count = (size_t)r * (size_t)c;
            w.off = off;
            w.layer = (int)li;
            off += w.count;
            s.weights.push_back(w);
        };
        if (l.kind == "dense") {
            long long a = l.geti("in", -1), b = l.geti("out", -1);
            if (a <= 0 || b <= 0) { err = "dense " + l.name + ": in= and out= required"; return false; }
            if (act_code(l.gets("act", "identity")) < 0) { err = "dense " + l.name + ": unknown act"; return false; }
            add(l.name + "_w", a, b);
        } else if (l.kind == "embedding") {
            long long v = l.geti("vocab", -1), d = l.geti("dim", -1);
            if (v <= 0 || d <= 0) { err = "embedding " + l.name + ": vocab= and dim= required"; return false; }
            add(l.name + "_w", v, d);
        } else if (l.kind == "attention") {
            long long d = l.geti("dim", -1), h = l.geti("heads", -1);
            if (d <= 0 || h <= 0 || d % h) { err = "attention " + l.name + ": dim divisible by heads"; return false; }
            for (const char* t : {"_q_w", "_k_w", "_v_w", "_o_w"}) add(l.name + t, d, d);
        } else if (l.kind == "moe") {
            long long d = l.geti("dim", -1), e = l.geti("experts", -1), f = l.geti("ffn", 4 * d);
            if (d <= 0 || e <= 0) { err = "moe " + l.name + ": dim= and experts= required"; return false; }
            add(l.name + "_g_w", d, e);
            if (l.gets("expert", "ffn") == "linear") {
                add(l.name + "_e1_w", e, d * d);
            } else {
                add(l.name + "_e1_w", e, d * f);
                add(l.name + "_e2_w", e, f * d);
            }
        } else if (l.kind == "dropout") {
            double r = 0.0;
            try { r = std::stod(l.gets("rate", "0")); } catch (...) { r = -1.0; }
            if (!(r >= 0.0 && r < 1.0)) { err = "dropout " + l.name + ": rate must be in [0, 1)"; return false; }
        } else if (l.kind == "layernorm") {
        } else {
            err = "unknown layer kind " + l.kind;
            return false;
        }
    }
    s.total = off;

    // widths along the graph
    s.width["x"] = s.in_cols;
    for (auto& op : s.ops) {
        if (op.args.empty()) { err = "op " + op.out + " has no arguments"; return false; }
        for (auto& a : op.args)
            if (!s.width.count(a)) { err = "op " + op.out + ": unknown value " + a; return false; }
        int w0 = s.width[op.args[0]];
        if (op.fn == "add" || op.fn == "sub" || op.fn == "mul" || op.fn == "div") {
            if (op.args.size() != 2) { err = op.fn + " takes two values"; return false; }
            if (s.width[op.args[1]] != w0) { err = op.out + ": width mismatch"; return false; }
            s.width[op.out] = w0;
        } else if (act_code(op.fn) >= 0 || op.fn == "softmax") {
            s.width[op.out] = w0;
        } else if (op.fn == "concat") {
            s.width[op.out] = w0 + s.width[op.args[1]];
        } else if (op.fn == "slice") {
            if (op.ints.size() != 2 || op.ints[0] < 0 || op.ints[1] > w0 || op.ints[1] <= op.ints[0]) {
                err = op.out + ": slice(u, cs, ce) needs 0 <= cs < ce <= width";
                return false;
            }
            s.width[op.out] = (int)(op.ints[1] - op.ints[0]);
        } else if (op.fn == "index" || op.fn == "scatter") {
            if (op.ints.empty()) { err = op.out + ": " + op.fn + " needs at least one column index"; return false; }
            for (long long c : op.ints)
                if (c < 0 || c >= w0) { err = op.out + ": column index out of range"; return false; }
            if (op.fn == "scatter" && s.width[op.args[1]] != (int)op.ints.size()) {
                err = op.out + ": scatter update width must equal the number of indices";
                return false;
            }
            s.width[op.out] = op.fn == "index" ? (int)op.ints.size() : w0;
        } else {
            int li = s.layer_index(op.fn);
            if (li < 0) { err = "unknown layer or function " + op.fn; return false; }
            const LayerSpec& l = s.layers[li];
            if (l.kind == "dense") {
                if (w0 != l.geti("in", 0)) { err = op.out + ": dense input width mismatch"; return false; }
                s.width[op.out] = (int)l.geti("out", 0);
            } else if (l.kind == "embedding") {
                if (!(op.args[0] == "x" && s.tokens)) { err = op.out + ": embedding reads the token input x"; return false; }
                s.width[op.out] = (int)l.geti("dim", 0);
            } else if (l.kind == "attention" || l.kind == "moe") {
                if (w0 != l.geti("dim", 0)) { err = op.out + ": width mismatch"; return false; }
                s.width[op.out] = w0;
            } else {
                s.width[op.out] = w0;
            }
        }
    }
    if (!s.width.count(s.output)) { err = "unknown output value " + s.output; return false; }
    s.out_cols = s.width[s.output];
    for (auto& w : s.weights) {
        ns_weight_desc d;
        d.name = w.name.c_str();
        d.offset = w.off;
        d.count = w.count;
        s.desc.push_back(d);
    }
    s.layout.num_weights = s.desc.size();
    s.layout.desc = s.desc.data();
    return true;
}

}  // namespace nsb
