/*
 * minigo_cuda.h - C ABI of the B200 network-evaluation backend.
 *
 * One handle = one network resident on one GPU, evaluated on that GPU's own
 * stream.  Calls on one handle must be serialised by the caller, exactly as
 * the reference's engines require (include/opencl_engine.h:24: one
 * NNEvaluator server thread drives one engine).  Every call returns 0 on
 * success or a negative MG_E* code; mg_last_error() then holds a message.
 * Nothing throws across this boundary.
 *
 * Semantics follow the reference interface include/inference_engine.h:
 * input states are 17 planes x board^2 fp32 values per position, plane-major
 * (src/game.cpp:229-256); outputs are softmax probabilities over
 * board^2 + 1 actions and a tanh value in [-1, 1] per position.
 */
#ifndef MINIGO_CUDA_H
#define MINIGO_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct mg_engine mg_engine;

/* Error codes. */
#define MG_OK 0
#define MG_E_ARG (-1)      /* bad argument (null pointer, size out of range)  */
#define MG_E_MODEL (-2)    /* model file or tensor set rejected                */
#define MG_E_CUDA (-3)     /* CUDA runtime or driver call failed               */
#define MG_E_STATE (-4)    /* call not valid in this state (no model loaded)   */
#define MG_E_DEVICE (-5)   /* a kernel reported an error (bounded wait expired) */

/* Arithmetic of the trunk (mg_set_precision). */
#define MG_PREC_BF16 0     /* bf16 operands, fp32 accumulate (tcgen05)        */
#define MG_PREC_FP16 1     /* fp16 operands, fp32 accumulate (tcgen05)        */
#define MG_PREC_FP32 2     /* fp32 SIMT verification path                     */

/* mg_create flags. */
#define MG_FLAG_EIGEN_COMPAT 1 /* read inputs and flatten the policy features
                                  the way src/eigen_engine.cpp:211,242 do
                                  (column-major Map), instead of the NCHW
                                  semantics of scripts/model.py:48-62        */

/* A named fp32 host tensor, as produced by any ONNX initializer parser
 * (replaces onnx_parser::OnnxTensor, include/onnx_loader.h:13-30). */
typedef struct mg_tensor {
    const char* name;
    const int64_t* dims;
    int ndims;
    const float* data; /* product(dims) little-endian fp32 values */
} mg_tensor;

/* Creates an engine on CUDA device `device`.  Replaces the backend
 * constructor called by create_engine() (src/inference_engine.cpp:16-24);
 * the device index is new (one engine per GPU).  Returns NULL on failure;
 * mg_create_error() then describes why. */
mg_engine* mg_create(int device, int flags);
const char* mg_create_error(void);

/* Releases every device and pinned host allocation of the engine. */
void mg_destroy(mg_engine* e);

/* Message describing the last failed call on this handle ("" if none). */
const char* mg_last_error(const mg_engine* e);

/* Loads weights from an ONNX file (initializers only).  Replaces
 * InferenceEngine::load_model (include/inference_engine.h:19) as implemented
 * by EigenEngine::load_from_onnx (src/eigen_engine.cpp:17-121): the
 * architecture is inferred from tensor names and shapes and BatchNorm is
 * folded with eps = 1e-5.  Errors name the file or the missing tensor. */
int mg_load_onnx(mg_engine* e, const char* path);

/* Same as mg_load_onnx for tensors already parsed by the caller (for example
 * by the reference's onnx_parser::parse_onnx_file, src/onnx_loader.cpp:183). */
int mg_load_weights(mg_engine* e, const mg_tensor* tensors, int count);

/* Model metadata, set by a successful load (include/inference_engine.h:36-40).
 * Any output pointer may be NULL. */
int mg_get_info(const mg_engine* e, int* board_size, int* input_channels,
                int* num_filters, int* num_res_blocks, int* action_size);

/* Selects MG_PREC_*.  Default MG_PREC_BF16. */
int mg_set_precision(mg_engine* e, int precision);

/* Largest positions per device launch (default 1024).  Larger batches are
 * evaluated in chunks.  Must be called before the first forward. */
int mg_set_max_batch(mg_engine* e, int max_batch);

/* Evaluates n positions held in HOST memory.  Replaces predict_batch
 * (include/inference_engine.h:25-32; src/opencl_engine.cpp:722-857) and, for
 * n = 1, predict (include/inference_engine.h:21-23).
 *   states      n x input_channels x board^2 fp32, position-major
 *   policy_out  n x action_size softmax probabilities
 *   value_out   n tanh values
 *   logits_out  n x action_size pre-softmax logits, or NULL
 * n == 0 is valid and does nothing (src/opencl_engine.cpp:724).
 * Blocks until the results are in the output buffers.  Pinned (page-locked)
 * host buffers are copied by DMA directly; pageable ones are staged. */
int mg_forward(mg_engine* e, const float* states, int n, float* policy_out,
               float* value_out, float* logits_out);

/* Bit-packed wire format.  The 17 input planes are binary, so a position can
 * travel as words_per_position = ceil(17 * board^2 / 32) little-endian
 * 32-bit words: element j of the plane-major state (c * board^2 + p) is bit
 * (j % 32) of word j / 32.  That is 768 bytes instead of 24.5 KB per 19x19
 * position on the host-to-device link.  No counterpart in the reference,
 * whose engines take fp32 planes (include/inference_engine.h:21-32). */
int mg_words_per_position(const mg_engine* e);

/* Packs n states of state_size fp32 values (each exactly 0 or 1) into
 * n * ceil(state_size / 32) words.  Returns MG_E_ARG if a value is neither
 * 0 nor 1 (such inputs need mg_forward).  Host-only; no engine needed. */
int mg_pack_states(const float* states, int n, int state_size, uint32_t* out);

/* As mg_forward for bit-packed inputs (n * mg_words_per_position words in
 * host memory; pinned buffers are copied by DMA directly).  Results are
 * identical to mg_forward on the unpacked planes. */
int mg_forward_packed(mg_engine* e, const uint32_t* bits, int n, float* policy_out,
                      float* value_out, float* logits_out);

/* Asynchronous form of mg_forward_packed for a batching server that
 * overlaps the host work of one batch (gathering its inputs, waking the
 * clients of the last one) with the GPU work of another: enqueues the copy
 * of n (<= mg_max_batch) bit-packed positions, the forward pass and the
 * copies of the results into policy_out / value_out on the engine's stream,
 * and returns at once with a ticket.  All three buffers must be page-locked
 * (mg_host_alloc); the input may be reused, and the outputs read, only after
 * mg_wait_submitted(ticket).  At most two submissions may be outstanding;
 * submissions complete in order.  mg_wait_submitted blocks until that
 * submission's results are in the output buffers and returns MG_OK,
 * MG_E_DEVICE if a kernel gave up waiting, or MG_E_ARG / MG_E_CUDA; it does
 * not set mg_last_error, and one thread may call it while another submits.
 * No counterpart in the reference, whose engines are synchronous. */
int mg_submit_packed(mg_engine* e, const uint32_t* bits, int n, float* policy_out,
                     float* value_out, int* ticket);
int mg_wait_submitted(mg_engine* e, int ticket);

/* History wire format: a position travels as the board-history ring that
 * GoGame::encode reads (src/game.cpp:213-256), and the 17 input planes are
 * expanded on the device.  mg_history_words(e) = 1 + 8 * ceil(board^2 / 16)
 * little-endian 32-bit words per position (185 words, 740 bytes, on 19x19):
 *   word 0: bits 0-1 the player to move (1 black, 2 white), bits 4-7 the
 *           number h of valid boards (0..8), bits 8-10 the ring slot `top`
 *           of the current board;
 *   then 8 slots of ceil(board^2 / 16) words; point p of a slot is at bits
 *           2 * (p % 16) .. +1 of word p / 16 (0 empty, 1 black, 2 white).
 * The board i moves back (i < h) is slot (top - i) mod 8.  Plane i (< 8)
 * marks the player to move's stones on it, plane 8 + i the opponent's;
 * plane 16 is all ones when black is to move.  A host that keeps its ring
 * in this packing ships it with one copy, with no per-evaluation encode.
 * Replaces the host-side GoGame::encode of src/mcts.cpp:206-209; results are
 * identical to mg_forward on the planes that encode writes.  Needs a
 * network with 17 input planes (MG_E_ARG otherwise). */
int mg_history_words(const mg_engine* e);
int mg_forward_history(mg_engine* e, const uint32_t* history, int n, float* policy_out,
                       float* value_out, float* logits_out);

/* The engine's pinned (page-locked) host input buffer, room for
 * mg_max_batch() positions.  Filling it and passing it to mg_forward avoids
 * any intermediate host copy.  Valid until mg_set_max_batch,
 * mg_set_precision, a new load or mg_destroy; NULL (see mg_last_error) if no
 * model is loaded or allocation fails. */
float* mg_host_input(mg_engine* e);

/* The same for the bit-packed wire format of mg_forward_packed: room for
 * mg_max_batch() positions of mg_words_per_position() words.  A batch
 * gathered here and passed to mg_forward_packed crosses to the device with
 * no intermediate host copy.  Same validity as mg_host_input.  No reference
 * counterpart (the reference ships fp32 planes). */
uint32_t* mg_host_bits(mg_engine* e);

/* Page-locked host memory of `bytes` bytes, for callers that keep their own
 * input or output buffers (a batching server's result slots): copies to and
 * from it are direct DMA instead of a staged copy through pageable memory.
 * NULL if the allocation fails.  Free with mg_host_free.  No reference
 * counterpart. */
void* mg_host_alloc(size_t bytes);
void mg_host_free(void* p);

/* Current max batch (mg_set_max_batch). */
int mg_max_batch(const mg_engine* e);

/* As mg_forward, with every pointer in this engine's device memory.
 * Enqueues on the engine's stream and returns without waiting; pair with
 * mg_synchronize.  n must not exceed the max batch. */
int mg_forward_device(mg_engine* e, const float* d_states, int n, float* d_policy,
                      float* d_value, float* d_logits);

/* As mg_forward_device, but allocates nothing: every intermediate buffer
 * comes from a fixed 32 MiB per-device scratch arena compiled into this
 * library, so it suits callers that may not call cudaMalloc/cudaFree once
 * running (both synchronise the device; cudaFree waits for all of it) or
 * that work inside a fixed GPU memory budget.  No counterpart in the
 * reference.  Limits: n is capped by the arena (19x19 bf16: 70 positions
 * with 128 filters, 37 with 256; the error message states the cap); the first call on
 * a device looks up the arena's address and should come before any stream
 * capture; all calls on a device share the arena, so calls whose work
 * overlaps on the GPU race and must be serialised.  Each call synchronises
 * the engine's stream before it returns (it reads the arena's status word
 * back to the host), so the results are in the output buffers on return;
 * d_logits may be NULL. */
int mg_forward_device_noalloc(mg_engine* e, const float* d_states, int n, float* d_policy,
                              float* d_value, float* d_logits);

/* Waits for all work on the engine's stream and reports device-side errors. */
int mg_synchronize(mg_engine* e);

/* The engine's cudaStream_t, for callers that time its work with events. */
void* mg_stream(mg_engine* e);

/* Launches `reps` back-to-back passes of one residual-block 3x3 convolution
 * layer (layer index 0 .. 2*blocks-1) over the activations left by the last
 * mg_forward_device of n positions.  A measurement hook: it lets a caller
 * time the trunk's convolution kernel alone with events on mg_stream(). */
int mg_launch_conv(mg_engine* e, int n, int layer, int reps);

/* Launches `reps` back-to-back passes of the whole trunk (every 3x3
 * convolution layer, as one persistent kernel where the engine uses one)
 * over the activations left by the last mg_forward_device of n positions.
 * A measurement hook like mg_launch_conv; no reference counterpart. */
int mg_launch_trunk(mg_engine* e, int n, int reps);

/* Number of kernel launches one mg_forward_device of n positions makes. */
int mg_launches_per_forward(mg_engine* e, int n);

#ifdef __cplusplus
}
#endif

#endif /* MINIGO_CUDA_H */
