// ORACLE - test infrastructure only.  A thin extern "C" harness around the
// reference's own sources, compiled unmodified from the reference tree by
// oracle/Makefile into oracle/_ref/libref_harness.so:
//   src/game.cpp        GoGame rules and encoder (position generation)
//   src/onnx_loader.cpp onnx_parser::parse_onnx_file
// Used by tests to pin the product's position generator and ONNX reader
// against the reference implementations.
#include "game.h"
#include "onnx_loader.h"

#include <cstdint>
#include <cstring>
#include <exception>
#include <random>
#include <string>
#include <vector>

using namespace minigo;

namespace {
uint32_t draw_below(uint32_t r, uint32_t range) {
    return (uint32_t)(((uint64_t)r * (uint64_t)range) >> 32);
}
std::vector<onnx_parser::OnnxTensor> g_tensors;
}  // namespace

extern "C" {

// The random-playout procedure of include/minigo_host.h, driven through the
// reference GoGame (is_legal src/game.cpp:164, play :176, encode :229).
int ref_random_positions(int board, int n, uint32_t seed, int max_moves, float* out) {
    std::mt19937 rng(seed);
    const int nn = board * board;
    const size_t per = (size_t)17 * nn;
    std::vector<int> legal;
    std::vector<float> enc;
    for (int i = 0; i < n; ++i) {
        GoGame g(board, 7.5f);
        const int k = (int)draw_below(rng(), (uint32_t)max_moves + 1u);
        for (int m = 0; m < k && !g.game_over; ++m) {
            legal.clear();
            for (int a = 0; a < nn; ++a)
                if (g.is_legal(a)) legal.push_back(a);
            legal.push_back(nn);
            g.play(legal[draw_below(rng(), (uint32_t)legal.size())]);
        }
        g.encode(enc);
        if (enc.size() != per) return -1;
        std::memcpy(out + (size_t)i * per, enc.data(), per * sizeof(float));
    }
    return 0;
}

// Parses a file with the reference loader; returns the tensor count or -1.
int ref_onnx_load(const char* path) {
    try {
        g_tensors = onnx_parser::parse_onnx_file(path);
        return (int)g_tensors.size();
    } catch (const std::exception&) {
        g_tensors.clear();
        return -1;
    }
}

const char* ref_onnx_name(int i) { return g_tensors.at(i).name.c_str(); }

int ref_onnx_dims(int i, int64_t* dims, int cap) {
    const auto& d = g_tensors.at(i).dims;
    for (int k = 0; k < (int)d.size() && k < cap; ++k) dims[k] = d[k];
    return (int)d.size();
}

int64_t ref_onnx_floats(int i, float* out, int64_t cap) {
    std::vector<float> v = g_tensors.at(i).get_floats();
    const int64_t k = cap < (int64_t)v.size() ? cap : (int64_t)v.size();
    if (k > 0) std::memcpy(out, v.data(), (size_t)k * sizeof(float));
    return (int64_t)v.size();
}

}  // extern "C"
