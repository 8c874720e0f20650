// Host-side network description built from named fp32 tensors.
//
// Architecture inference follows src/eigen_engine.cpp:84-95:
//   input_channels / filters from input_conv.weight [C, Cin, 3, 3];
//   blocks = number of consecutive res_blocks.{i}.conv1.weight names;
//   actions from policy_fc.weight [A, 2*B*B]; board = (int)sqrt(A - 1).
// BatchNorm is folded with eps = 1e-5 into a per-channel scale and bias
// exactly as src/eigen_engine.cpp:52-67 does (fp32 arithmetic, same order).
// Missing tensors raise std::runtime_error("Missing tensor: <name>")
// (src/eigen_engine.cpp:30); shape mismatches raise a message naming the
// tensor.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace mgb {

struct TensorView {
    std::string name;
    std::vector<int64_t> dims;
    const float* data = nullptr;  // product(dims) values
    size_t count = 0;             // number of values available at data
};

struct FoldedBn {
    std::vector<float> scale, bias;
};

struct HostConv {
    int cout = 0, cin = 0;
    std::vector<float> w;  // [cout][cin][3][3] as stored (unscaled)
    FoldedBn bn;
};

struct HostNet {
    int board = 0, input_channels = 0, filters = 0, blocks = 0, actions = 0, hidden = 0;
    HostConv input;
    std::vector<HostConv> conv1, conv2;  // per residual block
    std::vector<float> pconv_w;          // [2][C]
    FoldedBn pbn;                        // 2 channels
    std::vector<float> pfc_w, pfc_b;     // [A][2*B*B], [A]
    std::vector<float> vconv_w;          // [1][C]
    FoldedBn vbn;                        // 1 channel
    std::vector<float> v1_w, v1_b;       // [H][B*B], [H]
    std::vector<float> v2_w, v2_b;       // [1][H], [1]
};

// Builds the network; when a name repeats in `tensors`, the last one wins.
HostNet build_host_net(const std::vector<TensorView>& tensors);

// BN fold of src/eigen_engine.cpp:52-67.
FoldedBn fold_bn(const std::vector<float>& gamma, const std::vector<float>& beta,
                 const std::vector<float>& mean, const std::vector<float>& var);

}  // namespace mgb
