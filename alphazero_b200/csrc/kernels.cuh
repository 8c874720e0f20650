// Launch interfaces of the device kernels of the network-evaluation path.
//
// Activation layout ("framed NHWC"): a batch of positions on a board of side
// B is stored as rows of channel vectors, one row per pixel of a
// (B+1) x (B+1) frame per position: row = n*IS + y*RS + x with RS = B + 1,
// IS = RS * RS, or more (rows past RS * RS are zero padding).  Column x = B and row y = B of every frame are zero, so the
// 3x3 neighbour (y+dy, x+dx) of any board pixel is the row
// row + dy*RS + dx and reads zero whenever it falls off the board (the
// zero padding of src/eigen_engine.cpp:139-168); the rows before the first
// frame read as zero through TMA out-of-bounds fill.  Every kernel that
// writes activations writes zeros on frame pixels.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace mgb {

struct FrameGeom {
    int board;  // B
    int rs;     // B + 1
    int is;     // (B + 1)^2
};

// pad_to > 1: the frame stride rounded up to a multiple of pad_to rows; the
// extra rows at the end of each frame are frame pixels (zero) like the
// frame's last row and column.
inline FrameGeom make_frame(int board, int pad_to = 1) {
    FrameGeom g;
    g.board = board;
    g.rs = board + 1;
    g.is = ((board + 1) * (board + 1) + pad_to - 1) / pad_to * pad_to;
    return g;
}

// One 3x3 convolution layer, stride 1, zero padding 1, with folded
// BatchNorm bias, optional residual add and ReLU:
//   y[r, co] = relu(sum_{tap, ci} in[r + off(tap), ci] * W[co, tap, ci]
//                   + bias[co] (+ res32[r, co]))     on board pixels,
//   y[r, co] = 0                                     on frame pixels,
// written as fp32 to out32 and/or as the 16-bit operand type to out16.
// The residual stream is kept in fp32 (res32 / out32) so 16-bit rounding
// enters only through the tensor-core operands, not the running sum.  The
// 128-channel kernel keeps it instead as a 16-bit pair (res_hi + res_lo ->
// out16 + out_lo, below): about 20 significant bits in 4 bytes, of which the
// hi half is at once the next layer's operand.
//
// Optional fused head projection (tensor-core path, when one tile spans all
// output channels): for each board pixel p of position n,
//   feat[n][c*hw + p] = relu(sum_co y[r, co] * head_w[c][co] + head_b[c])
// for c = 0, 1 (policy) and c = 2 (value): the policy and value 1x1
// convolutions with folded BN and ReLU (src/eigen_engine.cpp:237-241,
// :257-260), laid out as the policy features in c*hw + p order followed by
// the value features.
struct ConvLayer {
    int m_total;            // rows = positions * IS
    int cin;                // input channels (multiple of 64)
    int cout;               // output channels (multiple of 64)
    FrameGeom g;
    const void* in;         // [m_total][cin], operand type
    const void* weight;     // [cout][9][cin], operand type
    const float* bias;      // [cout]
    const float* res32;     // [m_total][cout] fp32 or nullptr (may equal out32)
    float* out32;           // [m_total][cout] fp32 or nullptr
    void* out16;            // [m_total][cout] 16-bit or nullptr (tensor-core path)
    // Residual stream as a 16-bit pair (128-channel kernel only): x = hi + lo,
    // hi = x rounded to the operand type (the next layer reads it as its
    // input), lo = the remainder x - hi rounded to fp16.
    const void* res_hi;     // [m_total][cout] operand type or nullptr (may equal out16)
    // lo is stored in 16-pixel blocks, element (px, c) at
    // (px / 16) * 16 * cout + c * 16 + px % 16, rows rounded up to 16.
    const uint16_t* res_lo; // fp16, 16-pixel blocks (may equal out_lo)
    uint16_t* out_lo;       // fp16 remainder of out16, 16-pixel blocks, or nullptr
    const float* head_w;    // [3][cout] or nullptr: fused head projection
    const float* head_b;    // [3]
    float* feat;            // [positions][3*B*B]
    int* err;               // device status word
};

// Tensor-core path (bf16 or fp16 operands, fp32 accumulation in TMEM).
// tmA / tmB must describe layer.in / layer.weight (see make_conv_tensor_maps).
// bn = output channels per tile (64, 128 or 256; must divide cout).
cudaError_t launch_conv_tc(const ConvLayer& layer, const CUtensorMap& tmA, const CUtensorMap& tmB,
                           int bn, bool fp16, int grid_limit, cudaStream_t stream);

// The trunk layers of a 64/128/256-channel network (input conv first) as one
// persistent cooperative launch of the tensor-core kernel, with the schedule
// and cross-CTA progress counters of launch_trunk_pix (one tile spans every
// output channel; 128-row tiles).  Layers 1..n-1 must have cin == cout and
// their weights back to back from layers[1].weight; n <= trunk_tc_max_layers();
// progress points at grid_limit counters of scratch.  withhold_cta is the
// same failure-path test hook as launch_trunk_pix's.
bool trunk_tc_supported(const ConvLayer* layers, int n);
cudaError_t launch_trunk_tc(const ConvLayer* layers, int n, bool fp16, int grid_limit,
                            unsigned* progress, cudaStream_t stream, int withhold_cta = -1);
int trunk_tc_max_layers();

// cuTensorMapEncodeTiled of a dense 2-D [rows][inner] tensor of esize-byte
// elements, memoised per host thread.  The launchers encode the same maps
// at every launch (an encode costs microseconds of host time, which made
// launch-bound paths host-bound); a map depends only on these arguments, so
// a remembered one is exact.
bool encode_tiled_2d(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* base,
                     uint64_t inner, uint64_t rows, uint32_t box_inner, uint32_t box_rows,
                     CUtensorMapSwizzle swizzle);

// Host-side encoding of the two TMA descriptors of a layer.
bool make_conv_tensor_maps(const ConvLayer& layer, int bn, bool fp16, CUtensorMap* tmA,
                           CUtensorMap* tmB, const char** why);

// Shared-memory bytes the tensor-core kernel needs for a tile width bn on a
// board with row stride rs.
int conv_tc_smem_bytes(int bn, int rs);

// Sets the shared-memory opt-in of every tensor-core kernel instantiation on
// the current device (a per-device attribute; call once per device before
// launching or capturing).
cudaError_t configure_conv_tc();

// Tensor-core path for 128 output channels with pixels on the MMA N side
// (conv_pix.cu): each of up to grid_limit CTAs takes an equal contiguous
// pixel range cut into tiles of at most max_npx (<= 256) pixels; one halo
// slab per 64-channel block is shared by the 9 taps.
bool conv_pix_supported(const ConvLayer& layer, int npx);
cudaError_t launch_conv_pix(const ConvLayer& layer, int max_npx, bool fp16, int grid_limit,
                            cudaStream_t stream);
cudaError_t configure_conv_pix();

// The n trunk layers of a network (input conv first) as one persistent
// cooperative launch of the same kernel (several launches past 44 layers):
// each CTA keeps its pixel range through all layers and starts a tile of the
// next layer as soon as the tiles of the previous layer that it reads are
// stored.  Layers 1..n-1 must have cin 128 and their weights back to back
// from layers[1].weight; progress points at grid_limit counters of scratch.
// When CTAs get fewer than min_tiles tiles the layers go out as one launch
// each.  With own_frames (frames of whole 16-row chunks that fit one tile,
// FrameGeom padded) each CTA takes whole frames and waits only on its own
// tiles: the layers go out as one launch at any batch.  Needs every
// activation buffer's frame rows zero from allocation on.
// withhold_cta >= 0 is a test hook for the failure path: that CTA never
// publishes its progress, so the CTAs waiting on it (itself included) give up
// after the bounded wait and report kErrWaitDep in the status word.
cudaError_t launch_trunk_pix(const ConvLayer* layers, int n, int max_npx, bool fp16,
                             int grid_limit, unsigned* progress, cudaStream_t stream,
                             int withhold_cta = -1, int min_tiles = 1, bool own_frames = false);
// Number of kernel launches launch_trunk_pix makes for n layers of m_total rows.
int trunk_pix_launches(int m_total, int n, int max_npx, int grid_limit, int min_tiles = 1,
                       bool own_frames = false);

// fp32 SIMT path used by the fp32 verification mode.
cudaError_t launch_conv_simt(const ConvLayer& layer, cudaStream_t stream);

// Input staging: n_valid positions of plane-major fp32 states (17 planes of
// B*B, src/game.cpp:229-256) -> framed NHWC rows of `cpad` channels of type
// T for `n_pos` positions (positions >= n_valid are zero).  With
// eigen_order, state element (c, p) is read from c + p*planes instead of
// c*B*B + p, the column-major reading of src/eigen_engine.cpp:211.
enum class ActType { BF16 = 0, FP16 = 1, FP32 = 2 };
cudaError_t launch_stage_input(const float* states, int n_valid, int n_pos, int planes,
                               const FrameGeom& g, int cpad, bool eigen_order, ActType t,
                               void* out, cudaStream_t stream);

// As launch_stage_input for the bit-packed wire format: position n's
// planes are words_per_pos 32-bit words, element j (plane-major) in bit
// j & 31 of word j >> 5.
cudaError_t launch_stage_bits(const uint32_t* bits, int words_per_pos, int n_valid, int n_pos,
                              int planes, const FrameGeom& g, int cpad, bool eigen_order, ActType t,
                              void* out, cudaStream_t stream);

// As launch_stage_input for the history wire format (mg_forward_history in
// include/minigo_cuda.h): position n's words_per_pos words are a header
// (bits 0-1 the player to move, 1 black / 2 white; bits 4-7 the number h of
// valid boards; bits 8-10 the ring slot of the current board) and
// kHistoryBoards slots of ceil(B*B / 16) words, point p at bits 2*(p % 16)
// of word p / 16 (0 empty, 1 black, 2 white); the board i moves back is slot
// (top - i) mod kHistoryBoards, for i < h.  The 17 planes GoGame::encode
// writes (src/game.cpp:229-256) are expanded on the device.
constexpr int kHistoryBoards = 8;
cudaError_t launch_stage_history(const uint32_t* hist, int words_per_pos, int n_valid, int n_pos,
                                 const FrameGeom& g, int cpad, bool eigen_order, ActType t, void* out,
                                 cudaStream_t stream);

// Head projection as a separate pass (fp32 SIMT path, or when the
// tensor-core tile does not span all channels): the 1x1 policy / value
// convolutions over an fp32 trunk [positions * IS][c] -> feat (see
// ConvLayer for the formula).
cudaError_t launch_head_projection(const float* trunk, int positions, int c, const FrameGeom& g,
                                   const float* head_w, const float* head_b, float* feat,
                                   cudaStream_t stream);

// Policy FC and value FC1 as one fp32 GEMM over the features
// feat[n] = [policy (2*hw) | value (hw)]:
//   out[n][o] = sum_k feat[n][k] * W[o][k] + b[o],  o < actions + hidden,
// where W = [[policy_fc.weight, 0], [0, value_fc1.weight]] (the zero blocks
// are skipped), then per position a max-subtracted softmax over the
// `actions` logits and value = tanh(value_fc2(relu(hidden))) (src/eigen_engine.cpp:243-269).
struct HeadFc {
    int hw, actions, hidden;
    const float* w;     // [actions + hidden][3*hw]
    const float* b;     // [actions + hidden]
    const float* v2_w;  // [hidden]
    const float* v2_b;  // [1]
};
// The FC sums run in kHeadsFcSplits fixed K slices; scratch holds their
// partial sums, and then (slice 0's rows) the finished FC outputs.
constexpr int kHeadsFcSplits = 6;
cudaError_t launch_heads_fc(const float* feat, const HeadFc& h, int positions,
                            float* scratch /* [kHeadsFcSplits][positions][actions + hidden] */,
                            float* probs,
                            float* logits, float* value, cudaStream_t stream);

}  // namespace mgb
