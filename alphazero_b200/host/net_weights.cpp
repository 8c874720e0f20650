#include "net_weights.h"

#include <cmath>
#include <stdexcept>
#include <unordered_map>

namespace mgb {
namespace {

struct Lookup {
    std::unordered_map<std::string, const TensorView*> by_name;

    explicit Lookup(const std::vector<TensorView>& ts) {
        for (const auto& t : ts) by_name[t.name] = &t;  // last one wins
    }

    bool has(const std::string& n) const { return by_name.count(n) != 0; }

    const TensorView& get(const std::string& n) const {
        auto it = by_name.find(n);
        if (it == by_name.end()) throw std::runtime_error("Missing tensor: " + n);
        return *it->second;
    }

    std::vector<float> values(const std::string& n, const std::vector<int64_t>& shape) const {
        const TensorView& t = get(n);
        if (t.dims != shape) {
            std::string want, got;
            for (auto d : shape) want += std::to_string(d) + ",";
            for (auto d : t.dims) got += std::to_string(d) + ",";
            throw std::runtime_error("Tensor " + n + " has shape [" + got + "], expected [" + want +
                                     "]");
        }
        size_t count = 1;
        for (auto d : shape) count *= (size_t)d;
        if (t.count < count || t.data == nullptr)
            throw std::runtime_error("Tensor " + n + " holds fewer values than its shape");
        return std::vector<float>(t.data, t.data + count);
    }
};

FoldedBn load_bn(const Lookup& L, const std::string& prefix, int64_t ch) {
    return fold_bn(L.values(prefix + ".weight", {ch}), L.values(prefix + ".bias", {ch}),
                   L.values(prefix + ".running_mean", {ch}), L.values(prefix + ".running_var", {ch}));
}

HostConv load_conv3(const Lookup& L, const std::string& w, const std::string& bn, int64_t cout,
                    int64_t cin) {
    HostConv c;
    c.cout = (int)cout;
    c.cin = (int)cin;
    c.w = L.values(w, {cout, cin, 3, 3});
    c.bn = load_bn(L, bn, cout);
    return c;
}

}  // namespace

FoldedBn fold_bn(const std::vector<float>& gamma, const std::vector<float>& beta,
                 const std::vector<float>& mean, const std::vector<float>& var) {
    const float eps = 1e-5f;
    FoldedBn f;
    f.scale.resize(gamma.size());
    f.bias.resize(gamma.size());
    for (size_t i = 0; i < gamma.size(); ++i) {
        const float inv_std = 1.0f / std::sqrt(var[i] + eps);
        f.scale[i] = gamma[i] * inv_std;
        f.bias[i] = beta[i] - gamma[i] * mean[i] * inv_std;
    }
    return f;
}

HostNet build_host_net(const std::vector<TensorView>& tensors) {
    Lookup L(tensors);
    HostNet net;
    const TensorView& iw = L.get("input_conv.weight");
    if (iw.dims.size() != 4 || iw.dims[2] != 3 || iw.dims[3] != 3)
        throw std::runtime_error("Tensor input_conv.weight must be [C, Cin, 3, 3]");
    const int64_t C = iw.dims[0], Cin = iw.dims[1];
    net.filters = (int)C;
    net.input_channels = (int)Cin;
    int nb = 0;
    while (L.has("res_blocks." + std::to_string(nb) + ".conv1.weight")) ++nb;
    net.blocks = nb;
    const TensorView& pw = L.get("policy_fc.weight");
    if (pw.dims.size() != 2) throw std::runtime_error("Tensor policy_fc.weight must be 2-D");
    const int64_t A = pw.dims[0];
    net.actions = (int)A;
    net.board = (int)std::sqrt((float)(A - 1));
    const int64_t B = net.board, HW = B * B;
    if (B < 1 || HW + 1 != A)
        throw std::runtime_error("policy_fc.weight rows must be board^2 + 1");

    net.input = load_conv3(L, "input_conv.weight", "input_bn", C, Cin);
    net.conv1.resize(nb);
    net.conv2.resize(nb);
    for (int i = 0; i < nb; ++i) {
        const std::string p = "res_blocks." + std::to_string(i);
        net.conv1[i] = load_conv3(L, p + ".conv1.weight", p + ".bn1", C, C);
        net.conv2[i] = load_conv3(L, p + ".conv2.weight", p + ".bn2", C, C);
    }
    net.pconv_w = L.values("policy_conv.weight", {2, C, 1, 1});
    net.pbn = load_bn(L, "policy_bn", 2);
    net.pfc_w = L.values("policy_fc.weight", {A, 2 * HW});
    net.pfc_b = L.values("policy_fc.bias", {A});
    net.vconv_w = L.values("value_conv.weight", {1, C, 1, 1});
    net.vbn = load_bn(L, "value_bn", 1);
    const TensorView& v1 = L.get("value_fc1.weight");
    if (v1.dims.size() != 2) throw std::runtime_error("Tensor value_fc1.weight must be 2-D");
    const int64_t H = v1.dims[0];
    net.hidden = (int)H;
    net.v1_w = L.values("value_fc1.weight", {H, HW});
    net.v1_b = L.values("value_fc1.bias", {H});
    net.v2_w = L.values("value_fc2.weight", {1, H});
    net.v2_b = L.values("value_fc2.bias", {1});
    return net;
}

}  // namespace mgb
