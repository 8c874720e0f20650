// extern "C" surface of libminigo_host.so (include/minigo_host.h).
#include "../../include/minigo_host.h"
#include "go_positions.h"
#include "onnx_reader.h"

#include <algorithm>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

struct mg_onnx_file {
    std::vector<mgb::NamedTensor> tensors;
};

namespace {
thread_local std::string g_onnx_error;
}

extern "C" {

int mg_random_positions(int board, int n, uint32_t seed, int max_moves, float* out) {
    if (board < 2 || board > mgb::kMaxBoard || n < 0 || max_moves < 0 || (n > 0 && out == nullptr))
        return -1;
    mgb::random_positions(board, n, seed, max_moves, out);
    return 0;
}

int mg_random_histories(int board, int n, uint32_t seed, int max_moves, uint32_t* out) {
    if (board < 2 || board > mgb::kMaxBoard || n < 0 || max_moves < 0 || (n > 0 && out == nullptr))
        return -1;
    mgb::random_histories(board, n, seed, max_moves, out);
    return 0;
}

int mg_history_words_for(int board) {
    return (board < 2 || board > mgb::kMaxBoard) ? 0 : mgb::history_words(board);
}

mg_onnx_file* mg_onnx_open(const char* path) {
    g_onnx_error.clear();
    if (path == nullptr) {
        g_onnx_error = "null path";
        return nullptr;
    }
    try {
        auto* f = new mg_onnx_file();
        f->tensors = mgb::read_onnx_initializers(path);
        return f;
    } catch (const std::exception& e) {
        g_onnx_error = e.what();
        return nullptr;
    }
}

const char* mg_onnx_error(void) { return g_onnx_error.c_str(); }

void mg_onnx_close(mg_onnx_file* f) { delete f; }

int mg_onnx_count(const mg_onnx_file* f) { return f ? (int)f->tensors.size() : 0; }

const char* mg_onnx_name(const mg_onnx_file* f, int i) {
    if (!f || i < 0 || i >= (int)f->tensors.size()) return nullptr;
    return f->tensors[i].name.c_str();
}

int mg_onnx_data_type(const mg_onnx_file* f, int i) {
    if (!f || i < 0 || i >= (int)f->tensors.size()) return -1;
    return f->tensors[i].data_type;
}

int mg_onnx_dims(const mg_onnx_file* f, int i, int64_t* dims, int cap) {
    if (!f || i < 0 || i >= (int)f->tensors.size()) return -1;
    const auto& d = f->tensors[i].dims;
    for (int k = 0; k < (int)d.size() && k < cap; ++k) dims[k] = d[k];
    return (int)d.size();
}

int64_t mg_onnx_floats(const mg_onnx_file* f, int i, float* out, int64_t cap) {
    if (!f || i < 0 || i >= (int)f->tensors.size()) return -1;
    try {
        std::vector<float> v = f->tensors[i].floats();
        const int64_t k = std::min<int64_t>(cap, (int64_t)v.size());
        if (k > 0) std::memcpy(out, v.data(), (size_t)k * sizeof(float));
        return (int64_t)v.size();
    } catch (const std::exception&) {
        return -1;
    }
}

}  // extern "C"
