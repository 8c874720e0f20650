/*
 * minigo_host.h - C ABI of the host-side (CPU-only) helpers that feed the
 * network-evaluation path: the seeded position generator and the ONNX
 * initializer reader.  Built as libminigo_host.so, which needs no GPU.
 */
#ifndef MINIGO_HOST_H
#define MINIGO_HOST_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Writes n positions of 17 x board^2 fp32 planes (the encoding of
 * GoGame::encode, src/game.cpp:229-256) to out.  Position i is reached from
 * the empty board by k_i uniformly random legal moves (pass included,
 * stopping if the game ends), k_i uniform in [0, max_moves]; all draws come
 * from one std::mt19937(seed) mapped by floor(r * range / 2^32).
 * Returns 0, or -1 for bad arguments (board outside 2..19, n < 0). */
int mg_random_positions(int board, int n, uint32_t seed, int max_moves, float* out);

/* The same positions in the history wire format of mg_forward_history
 * (include/minigo_cuda.h): mg_history_words_for(board) 32-bit words each.
 * No reference counterpart (the reference encodes planes on the host). */
int mg_random_histories(int board, int n, uint32_t seed, int max_moves, uint32_t* out);
int mg_history_words_for(int board);

/* ONNX initializer reader (replaces onnx_parser::parse_onnx_file,
 * src/onnx_loader.cpp:183-195). */
typedef struct mg_onnx_file mg_onnx_file;

/* Returns NULL on failure; mg_onnx_error() then holds the message (for a
 * missing file: "Cannot open model file: <path>", src/onnx_loader.cpp:186). */
mg_onnx_file* mg_onnx_open(const char* path);
const char* mg_onnx_error(void);
void mg_onnx_close(mg_onnx_file* f);
int mg_onnx_count(const mg_onnx_file* f);
const char* mg_onnx_name(const mg_onnx_file* f, int i);
int mg_onnx_data_type(const mg_onnx_file* f, int i);
/* Writes up to cap dims; returns the rank. */
int mg_onnx_dims(const mg_onnx_file* f, int i, int64_t* dims, int cap);
/* Writes up to cap fp32 values; returns how many the tensor holds, or -1 if
 * it is not FLOAT. */
int64_t mg_onnx_floats(const mg_onnx_file* f, int i, float* out, int64_t cap);

#ifdef __cplusplus
}
#endif

#endif /* MINIGO_HOST_H */
