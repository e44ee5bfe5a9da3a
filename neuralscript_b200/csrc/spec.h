// Model spec: parsed form of the text description a NeuralScript network
// lowers to (grammar in neuralscript_b200/spec.py). Weight names and blob
// order follow the reference's TENSOR_ALLOC order
// (src/mlir/mlir_compiler.cpp:100-222).
#pragma once
#include <map>
#include <string>
#include <vector>

#include "../../include/ns_runtime.h"

namespace nsb {

struct LayerSpec {
    std::string name, kind;
    std::map<std::string, std::string> p;
    long long geti(const std::string& k, long long def) const {
        auto it = p.find(k);
        return it == p.end() ? def : std::stoll(it->second);
    }
    std::string gets(const std::string& k, const std::string& def) const {
        auto it = p.find(k);
        return it == p.end() ? def : it->second;
    }
};

struct SpecOp {
    std::string out, fn;
    std::vector<std::string> args;  // value operands
    std::vector<long long> ints;    // integer operands (slice bounds, column indices)
};

// Data-movement functions and how many value operands they take before the
// integer operands: concat(a, b), slice(u, cs, ce), index(u, i0, ...),
// scatter(u, upd, i0, ...).
int data_fn_values(const std::string& fn);

struct WeightInfo {
    std::string name;
    size_t off = 0, count = 0;
    int rows = 0, cols = 0;
    int layer = -1;
};

struct Spec {
    std::string text;
    std::string name = "model";
    int in_cols = 1;
    bool tokens = false;
    std::vector<LayerSpec> layers;
    std::vector<SpecOp> ops;
    std::string output;
    std::string loss = "cross_entropy";
    std::string optimizer = "reference";
    std::map<std::string, double> opt;
    std::string schedule = "constant";
    std::map<std::string, double> sched;
    int precision = 2;  // 0 fp32, 1 tf32, 2 bf16
    bool input_grad = false;  // `grad input`: train steps also form dLoss/dx
    std::vector<WeightInfo> weights;
    size_t total = 0;
    std::map<std::string, int> width;  // value name -> columns
    int out_cols = 1;
    // ABI layout table (names point into `weights`)
    std::vector<ns_weight_desc> desc;
    ns_weight_layout layout{0, nullptr};

    int layer_index(const std::string& n) const {
        for (size_t i = 0; i < layers.size(); i++)
            if (layers[i].name == n) return (int)i;
        return -1;
    }
    const WeightInfo* weight(const std::string& n) const {
        for (auto& w : weights)
            if (w.name == n) return &w;
        return nullptr;
    }
    double optv(const std::string& k, double def) const {
        auto it = opt.find(k);
        return it == opt.end() ? def : it->second;
    }
    double schedv(const std::string& k, double def) const {
        auto it = sched.find(k);
        return it == sched.end() ? def : it->second;
    }
};

// Activation name -> code (0 identity .. 6 gelu), -1 if unknown.
int act_code(const std::string& name);

// Parses and validates; on failure returns false with a message.
bool parse_spec(const std::string& text, Spec& out, std::string& err);

}  // namespace nsb
