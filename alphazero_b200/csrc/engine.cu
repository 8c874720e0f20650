// The network-evaluation engine behind the C ABI of include/minigo_cuda.h.
//
// Load time (src/eigen_engine.cpp:17-121 semantics): named fp32 tensors ->
// HostNet (architecture inference + BN fold) -> device weights with the BN
// scale folded into each conv's output channels, reordered to
// [cout][tap][cin] with channels zero-padded to multiples of 64, in the
// trunk's arithmetic type; heads stay fp32.
//
// Run time, per batch of n positions (n <= max batch):
//   stage kernel (fp32 planes -> framed NHWC), then one CUDA graph per
//   batch-size bucket holding 1 + 2*blocks convolution launches and the heads
//   launch; host callers add one H2D copy before and D2H copies after, all on
//   the engine's own stream.  Positions between n and the bucket size are
//   computed on zero input and discarded.
#include "../../include/minigo_cuda.h"
#include "../host/net_weights.h"
#include "../host/onnx_reader.h"
#include "kernels.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

using namespace mgb;

namespace {

thread_local std::string g_create_error;

constexpr int kStagedChannels = 64;  // input planes padded to one 64-channel K block

int round_up(int v, int m) { return (v + m - 1) / m * m; }

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

struct CudaFailure {
    cudaError_t code;
    std::string where;
};

void ck(cudaError_t e, const char* where) {
    if (e != cudaSuccess) throw CudaFailure{e, where};
}

template <typename T>
T* dalloc(size_t count, const char* what) {
    void* p = nullptr;
    if (count == 0) count = 1;
    ck(cudaMalloc(&p, count * sizeof(T)), what);
    return reinterpret_cast<T*>(p);
}

}  // namespace

struct mg_engine {
    int device = 0;
    int flags = 0;
    int precision = MG_PREC_BF16;
    int max_batch = 1024;
    int num_sms = 148;
    int conv_bn_override = 0;
    int pix_mode = 1;      // 1: pixels-on-N kernel for 128-channel layers
    int pix_npx = 0;       // pixels per tile override (0 = heuristic)
    int pix_trunk = 1;     // 1: all 128-channel trunk layers as one persistent launch
    int pix_trunk_min_tiles = 1;  // ... when every CTA gets at least this many tiles
    // 1: 64/256-channel trunk layers as persistent launches.  Off by default:
    // measured no faster than one launch per layer (19x19 b20c256 batch
    // 1024: 0-1% slower, within the power-capped clock's noise; 9x9 b6c64
    // batch 16, one tile per CTA: 3% slower, 86 against 82 us per forward).
    int tc_trunk = 0;
    // 1: on boards whose frame fits one tile of the 128-channel kernel, pad
    // the frame stride to whole 16-row chunks and run the trunk as one
    // launch of CTAs that own whole frames (MG_FRAME_TRUNK=1).  Off by
    // default: bit-identical, and measured no faster at 9x9 batch 256
    // (trunk 250 us either way; 255 us with one frame per tile): with one
    // tile per CTA each layer's MMA, epilogue and publish run one after
    // another on every SM, and the launches and cross-CTA waits this
    // removes were not what that costs.
    int frame_trunk = 0;
    int withhold_cta = -1;  // test hook (MG_TEST_WITHHOLD_PROGRESS): see launch_trunk_pix
    bool use_graphs = true;
    // 1: keep the residual lo plane resident in L2 where it fits (default);
    // 2: mark it streaming (evict-first) instead; 0: no window
    // (MG_L2_POLICY).
    int l2_policy = 1;
    cudaStream_t stream = nullptr;
    std::string err;

    bool loaded = false;
    HostNet net;
    FrameGeom g{};
    int hw = 0, planes = 0, cpad = 0, actions = 0;
    int n_convs = 0;

    // Folded fp32 conv weights [cpad][9][cin_pad] and biases [cpad] (host).
    std::vector<std::vector<float>> wf;
    std::vector<int> wcin;  // cin_pad per conv
    std::vector<std::vector<float>> bf;

    // Device weights.
    std::vector<void*> d_w16;  // current 16-bit type (w16_prec), pointers into d_w16_all
    void* d_w16_all = nullptr;  // all layers' 16-bit weights, back to back
    int w16_prec = -1;
    std::vector<float*> d_w32;
    std::vector<float*> d_bias;
    float* d_head = nullptr;  // packed head parameters
    const float* d_head_w = nullptr;
    const float* d_head_b = nullptr;
    HeadFc fc{};

    // Device buffers for `alloc_batch` positions, element size `alloc_elem`.
    int alloc_batch = 0;
    int alloc_elem = 0;
    void* d_stage = nullptr;  // staged input rows, operand type
    float* d_x = nullptr;     // fp32 residual stream
    void* d_x16 = nullptr;    // 16-bit copy of d_x (tensor-core operand)
    // The 128-channel 16-bit path keeps the residual stream as d_x16 (hi) plus
    // an fp16 remainder plane (lo), which lives in d_x's storage there.
    void* d_t = nullptr;      // block-internal activation, operand type
    float* d_feat = nullptr;  // head features [positions][3*hw]
    float* d_fc = nullptr;    // FC partial sums [kHeadsFcSplits][positions][actions + hidden]
    float* d_states = nullptr;
    float* d_probs = nullptr;
    float* d_logits = nullptr;
    float* d_value = nullptr;
    int* d_err = nullptr;
    unsigned* d_progress = nullptr;  // [num_sms] per-CTA counters of the trunk kernel
    float* h_states = nullptr;  // pinned staging for pageable inputs
    int* h_err = nullptr;       // pinned status word
    uint32_t* d_bits = nullptr;  // bit-packed inputs [max_batch][words]
    uint32_t* h_bits = nullptr;  // pinned staging for pageable packed inputs
    uint32_t* d_hist = nullptr;  // history wire format inputs [max_batch][history_words()]
    uint32_t* h_hist = nullptr;  // pinned staging for pageable history inputs

    std::map<std::pair<int, int>, cudaGraphExec_t> graphs;  // (bucket, precision)
    int last_bucket = 0;

    // Submissions of mg_submit_packed: per ticket slot, an event recorded
    // after the results' copies and the status word copied back.
    static constexpr int kTickets = 4;
    cudaEvent_t tick_ev[kTickets] = {};
    int* h_tick_err = nullptr;  // pinned [kTickets]
    std::atomic<int> next_ticket{0};  // read by mg_wait_submitted on another thread

    ~mg_engine() { release_all(); }

    void drop_graphs() {
        for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
        graphs.clear();
    }

    void free_buffers() {
        drop_graphs();
        for (void* p : {d_stage, (void*)d_x, d_x16, d_t, (void*)d_feat, (void*)d_fc}) if (p) cudaFree(p);
        for (void* p : {(void*)d_states, (void*)d_probs, (void*)d_logits, (void*)d_value, (void*)d_err,
                        (void*)d_progress})
            if (p) cudaFree(p);
        d_progress = nullptr;
        if (h_states) cudaFreeHost(h_states);
        if (h_err) cudaFreeHost(h_err);
        if (h_tick_err) cudaFreeHost(h_tick_err);
        h_tick_err = nullptr;
        if (d_bits) cudaFree(d_bits);
        if (h_bits) cudaFreeHost(h_bits);
        if (d_hist) cudaFree(d_hist);
        if (h_hist) cudaFreeHost(h_hist);
        d_bits = nullptr;
        h_bits = nullptr;
        d_hist = nullptr;
        h_hist = nullptr;
        d_stage = d_x16 = d_t = nullptr;
        d_x = d_feat = d_fc = nullptr;
        d_states = d_probs = d_logits = d_value = nullptr;
        d_err = nullptr;
        h_states = nullptr;
        h_err = nullptr;
        alloc_batch = 0;
        alloc_elem = 0;
    }

    void free_weights() {
        drop_graphs();
        if (d_w16_all) cudaFree(d_w16_all);
        d_w16_all = nullptr;
        for (float* p : d_w32) if (p) cudaFree(p);
        for (float* p : d_bias) if (p) cudaFree(p);
        if (d_head) cudaFree(d_head);
        d_w16.clear();
        d_w32.clear();
        d_bias.clear();
        d_head = nullptr;
        w16_prec = -1;
    }

    void release_all() {
        DeviceGuard dg(device);
        free_buffers();
        free_weights();
        for (cudaEvent_t& ev : tick_ev)
            if (ev) {
                cudaEventDestroy(ev);
                ev = nullptr;
            }
        if (stream) cudaStreamDestroy(stream);
        stream = nullptr;
    }

    int elem_bytes() const { return precision == MG_PREC_FP32 ? 4 : 2; }
    int words_per_pos() const { return (planes * hw + 31) / 32; }
    // 32-bit words per position of the history wire format.
    int history_words() const { return 1 + kHistoryBoards * ((hw + 15) / 16); }
    ActType act_type() const {
        return precision == MG_PREC_FP32 ? ActType::FP32
                                         : (precision == MG_PREC_FP16 ? ActType::FP16 : ActType::BF16);
    }

    // ---- load ----------------------------------------------------------

    void load(const std::vector<TensorView>& views) {
        HostNet n = build_host_net(views);
        if (n.input_channels > kStagedChannels)
            throw std::runtime_error("input_conv.weight has " + std::to_string(n.input_channels) +
                                     " input channels; at most 64 are supported");
        if (n.filters > 256)
            throw std::runtime_error("num_filters " + std::to_string(n.filters) +
                                     " exceeds the supported maximum of 256");
        if (n.board > 25) throw std::runtime_error("board sizes above 25 are not supported");
        if (n.hidden > 1024) throw std::runtime_error("value_fc1 width above 1024 is not supported");
        free_weights();
        free_buffers();
        net = std::move(n);
        hw = net.board * net.board;
        planes = net.input_channels;
        cpad = round_up(net.filters, 64);
        g = make_frame(net.board);
        if (frame_trunk != 0 && cpad == 128 && g.is <= 256) g = make_frame(net.board, 16);
        actions = net.actions;
        n_convs = 1 + 2 * net.blocks;

        // Fold the BN scale into output channels; [cout][cin][3][3] ->
        // [cpad][tap][cin_pad].
        wf.assign(n_convs, {});
        bf.assign(n_convs, {});
        wcin.assign(n_convs, 0);
        auto fold = [&](int li, const HostConv& c, int cin_pad) {
            std::vector<float>& w = wf[li];
            w.assign((size_t)cpad * 9 * cin_pad, 0.0f);
            for (int co = 0; co < c.cout; ++co)
                for (int ci = 0; ci < c.cin; ++ci)
                    for (int tap = 0; tap < 9; ++tap)
                        w[((size_t)co * 9 + tap) * cin_pad + ci] =
                            c.w[((size_t)co * c.cin + ci) * 9 + tap] * c.bn.scale[co];
            bf[li].assign(cpad, 0.0f);
            for (int co = 0; co < c.cout; ++co) bf[li][co] = c.bn.bias[co];
            wcin[li] = cin_pad;
        };
        fold(0, net.input, kStagedChannels);
        for (int b = 0; b < net.blocks; ++b) {
            fold(1 + 2 * b, net.conv1[b], cpad);
            fold(2 + 2 * b, net.conv2[b], cpad);
        }

        DeviceGuard dg(device);
        d_bias.resize(n_convs, nullptr);
        for (int li = 0; li < n_convs; ++li) {
            d_bias[li] = dalloc<float>(cpad, "cudaMalloc(bias)");
            ck(cudaMemcpy(d_bias[li], bf[li].data(), cpad * sizeof(float), cudaMemcpyHostToDevice),
               "cudaMemcpy(bias)");
        }
        upload_heads();
        loaded = true;
        prepare_weights();
    }

    void upload_heads() {
        const int A = actions, H = net.hidden, C = cpad;
        // Head projection: folded 1x1 convs [3][C] (policy 0, policy 1, value).
        std::vector<float> hw3((size_t)3 * C, 0.0f), hb3(3);
        for (int c = 0; c < 2; ++c)
            for (int k = 0; k < net.filters; ++k)
                hw3[(size_t)c * C + k] = net.pconv_w[(size_t)c * net.filters + k] * net.pbn.scale[c];
        for (int k = 0; k < net.filters; ++k) hw3[(size_t)2 * C + k] = net.vconv_w[k] * net.vbn.scale[0];
        hb3[0] = net.pbn.bias[0];
        hb3[1] = net.pbn.bias[1];
        hb3[2] = net.vbn.bias[0];
        // FC block matrix over feat = [policy c*hw + p | value p]:
        // rows < A are policy_fc (its columns permuted from the column-major
        // flatten c + 2p of src/eigen_engine.cpp:242 under eigen_compat),
        // rows >= A are value_fc1.
        const int K = 3 * hw;
        std::vector<float> wcat((size_t)(A + H) * K, 0.0f), bcat(A + H);
        const bool eig = (flags & MG_FLAG_EIGEN_COMPAT) != 0;
        for (int a = 0; a < A; ++a) {
            for (int c = 0; c < 2; ++c)
                for (int p = 0; p < hw; ++p) {
                    const int src = eig ? (c + 2 * p) : (c * hw + p);
                    wcat[(size_t)a * K + c * hw + p] = net.pfc_w[(size_t)a * 2 * hw + src];
                }
            bcat[a] = net.pfc_b[a];
        }
        for (int j = 0; j < H; ++j) {
            for (int p = 0; p < hw; ++p) wcat[(size_t)(A + j) * K + 2 * hw + p] = net.v1_w[(size_t)j * hw + p];
            bcat[A + j] = net.v1_b[j];
        }
        std::vector<std::pair<const float*, size_t>> parts = {
            {hw3.data(), hw3.size()},   {hb3.data(), 3},           {wcat.data(), wcat.size()},
            {bcat.data(), bcat.size()}, {net.v2_w.data(), (size_t)H}, {net.v2_b.data(), 1}};
        std::vector<size_t> offs;
        size_t total = 0;
        for (auto& pr : parts) {
            offs.push_back(total);
            total += (pr.second + 63) / 64 * 64;  // 256-byte aligned pieces
        }
        std::vector<float> packed(total, 0.0f);
        for (size_t i = 0; i < parts.size(); ++i)
            std::memcpy(packed.data() + offs[i], parts[i].first, parts[i].second * sizeof(float));
        d_head = dalloc<float>(total, "cudaMalloc(heads)");
        ck(cudaMemcpy(d_head, packed.data(), total * sizeof(float), cudaMemcpyHostToDevice),
           "cudaMemcpy(heads)");
        d_head_w = d_head + offs[0];
        d_head_b = d_head + offs[1];
        fc.hw = hw;
        fc.actions = A;
        fc.hidden = H;
        fc.w = d_head + offs[2];
        fc.b = d_head + offs[3];
        fc.v2_w = d_head + offs[4];
        fc.v2_b = d_head + offs[5];
    }

    // Device weights in the current precision's type (16-bit for the tensor
    // cores, fp32 for the SIMT path).
    void prepare_weights() {
        DeviceGuard dg(device);
        if (precision == MG_PREC_FP32) {
            if (d_w32.empty()) {
                d_w32.resize(n_convs, nullptr);
                for (int li = 0; li < n_convs; ++li) {
                    d_w32[li] = dalloc<float>(wf[li].size(), "cudaMalloc(w32)");
                    ck(cudaMemcpy(d_w32[li], wf[li].data(), wf[li].size() * sizeof(float),
                                  cudaMemcpyHostToDevice),
                       "cudaMemcpy(w32)");
                }
            }
            return;
        }
        if (w16_prec == precision) return;
        drop_graphs();  // captured graphs hold the old weight pointers
        if (d_w16_all) cudaFree(d_w16_all);
        d_w16_all = nullptr;
        d_w16.assign(n_convs, nullptr);
        // One allocation, layers back to back (each layer's size is a
        // multiple of 16 bytes), as the persistent trunk kernel reads them.
        size_t total = 0;
        for (int li = 0; li < n_convs; ++li) total += wf[li].size();
        d_w16_all = dalloc<uint16_t>(total, "cudaMalloc(w16)");
        size_t off = 0;
        for (int li = 0; li < n_convs; ++li) {
            const size_t cnt = wf[li].size();
            std::vector<uint16_t> h(cnt);
            if (precision == MG_PREC_BF16) {
                for (size_t i = 0; i < cnt; ++i) {
                    __nv_bfloat16 v = __float2bfloat16_rn(wf[li][i]);
                    std::memcpy(&h[i], &v, 2);
                }
            } else {
                for (size_t i = 0; i < cnt; ++i) {
                    __half v = __float2half_rn(wf[li][i]);
                    std::memcpy(&h[i], &v, 2);
                }
            }
            d_w16[li] = static_cast<uint16_t*>(d_w16_all) + off;
            off += cnt;
            ck(cudaMemcpy(d_w16[li], h.data(), cnt * 2, cudaMemcpyHostToDevice), "cudaMemcpy(w16)");
        }
        w16_prec = precision;
    }

    // ---- buffers ---------------------------------------------------------

    void ensure_buffers() {
        const int elem = elem_bytes();
        if (alloc_batch == max_batch && alloc_elem >= elem) return;
        DeviceGuard dg(device);
        free_buffers();
        const size_t rows = (size_t)max_batch * g.is;
        d_stage = dalloc<uint8_t>(rows * kStagedChannels * elem, "cudaMalloc(stage)");
        d_x = dalloc<float>(rows * cpad, "cudaMalloc(act x)");
        d_x16 = dalloc<uint16_t>(rows * cpad, "cudaMalloc(act x16)");
        d_t = dalloc<uint8_t>(rows * cpad * elem, "cudaMalloc(act t)");
        // Frame rows start out zero (every layer keeps them so); the
        // whole-frame trunk schedule reads other CTAs' frame rows unordered.
        ck(cudaMemset(d_stage, 0, rows * kStagedChannels * elem), "cudaMemset(stage)");
        ck(cudaMemset(d_x, 0, rows * cpad * sizeof(float)), "cudaMemset(act x)");
        ck(cudaMemset(d_x16, 0, rows * cpad * 2), "cudaMemset(act x16)");
        ck(cudaMemset(d_t, 0, rows * cpad * elem), "cudaMemset(act t)");
        d_feat = dalloc<float>((size_t)max_batch * 3 * hw, "cudaMalloc(feat)");
        d_fc = dalloc<float>((size_t)kHeadsFcSplits * max_batch * (actions + net.hidden),
                             "cudaMalloc(fc)");
        d_states = dalloc<float>((size_t)max_batch * planes * hw, "cudaMalloc(states)");
        ck(cudaMemset(d_states, 0, (size_t)max_batch * planes * hw * sizeof(float)),
           "cudaMemset(states)");
        d_probs = dalloc<float>((size_t)max_batch * actions, "cudaMalloc(probs)");
        d_logits = dalloc<float>((size_t)max_batch * actions, "cudaMalloc(logits)");
        d_value = dalloc<float>((size_t)max_batch, "cudaMalloc(value)");
        d_err = dalloc<int>(1, "cudaMalloc(err)");
        d_progress = dalloc<unsigned>((size_t)num_sms, "cudaMalloc(progress)");
        ck(cudaMemset(d_err, 0, sizeof(int)), "cudaMemset(err)");
        ck(cudaMallocHost(reinterpret_cast<void**>(&h_states),
                          (size_t)max_batch * planes * hw * sizeof(float)),
           "cudaMallocHost(states)");
        ck(cudaMallocHost(reinterpret_cast<void**>(&h_err), sizeof(int)), "cudaMallocHost(err)");
        ck(cudaMallocHost(reinterpret_cast<void**>(&h_tick_err), kTickets * sizeof(int)),
           "cudaMallocHost(ticket status)");
        d_bits = dalloc<uint32_t>((size_t)max_batch * words_per_pos(), "cudaMalloc(bits)");
        ck(cudaMemset(d_bits, 0, (size_t)max_batch * words_per_pos() * 4), "cudaMemset(bits)");
        ck(cudaMallocHost(reinterpret_cast<void**>(&h_bits), (size_t)max_batch * words_per_pos() * 4),
           "cudaMallocHost(bits)");
        d_hist = dalloc<uint32_t>((size_t)max_batch * history_words(), "cudaMalloc(history)");
        ck(cudaMemset(d_hist, 0, (size_t)max_batch * history_words() * 4), "cudaMemset(history)");
        ck(cudaMallocHost(reinterpret_cast<void**>(&h_hist), (size_t)max_batch * history_words() * 4),
           "cudaMallocHost(history)");
        alloc_batch = max_batch;
        alloc_elem = elem;
        if (l2_policy != 0 && precision != MG_PREC_FP32) apply_l2_policy(rows * cpad * 2);
    }

    // The 16-bit paths' residual lo plane (in d_x's storage) is written by
    // one block's conv2 and read back by the next block's, two layers later;
    // the activations streamed in between (t and the hi plane) exceed the
    // 126 MB L2 and evict it.  An L2 access-policy window on the engine's
    // stream marks it persisting, in a set-aside of the L2 for persisting
    // lines (a limit of this process's CUDA context, released with it).
    // Measured at 19x19, 128 filters, batch 512: trunk 1015 -> 994 us.  Only
    // when the whole plane fits the set-aside: a window persisting 82 MB of
    // the 20-block 256-filter net's 210 MB plane at batch 1024 made its trunk
    // 26% slower.  Graphs captured on the stream keep the window in their
    // kernel nodes.
    void apply_l2_policy(size_t lo_bytes) {
        int max_persist = 0, max_window = 0;
        if (cudaDeviceGetAttribute(&max_persist, cudaDevAttrMaxPersistingL2CacheSize, device) !=
                cudaSuccess ||
            cudaDeviceGetAttribute(&max_window, cudaDevAttrMaxAccessPolicyWindowSize, device) !=
                cudaSuccess ||
            max_persist <= 0 || max_window <= 0) {
            cudaGetLastError();
            return;  // no persisting L2 on this device: nothing to do
        }
        const bool streaming = l2_policy == 2;  // evict-first, no set-aside
        if (!streaming && (lo_bytes > (size_t)max_persist || lo_bytes > (size_t)max_window)) return;
        const size_t window = std::min(lo_bytes, (size_t)max_window);
        const size_t set_aside = streaming ? 0 : std::min(window, (size_t)max_persist);
        if (set_aside > 0)
            ck(cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, set_aside),
               "cudaDeviceSetLimit(persisting L2)");
        cudaStreamAttrValue attr = {};
        attr.accessPolicyWindow.base_ptr = d_x;
        attr.accessPolicyWindow.num_bytes = window;
        attr.accessPolicyWindow.hitRatio = (float)((double)set_aside / (double)window);
        attr.accessPolicyWindow.hitProp = cudaAccessPropertyPersisting;
        attr.accessPolicyWindow.missProp = cudaAccessPropertyStreaming;
        ck(cudaStreamSetAttribute(stream, cudaStreamAttributeAccessPolicyWindow, &attr),
           "cudaStreamSetAttribute(access policy window)");
    }

    int bucket_for(int n) const {
        static const int kBuckets[] = {1,   2,   4,   8,   16,   32,   64,   96,   128,  192, 256,
                                       320, 384, 448, 512, 640, 768, 896, 1024, 1536, 2048};
        for (int b : kBuckets)
            if (b >= n) return std::min(b, max_batch);
        return max_batch;
    }

    int choose_bn(int m_total) const {
        if (conv_bn_override > 0 && cpad % conv_bn_override == 0) return conv_bn_override;
        int bn = std::min(cpad, 256);
        while (cpad % bn != 0) bn -= 64;
        const int mt = (m_total + 127) / 128;
        while (bn > 64 && (long)mt * (cpad / bn) < 2L * num_sms && cpad % (bn / 2) == 0 &&
               (bn / 2) % 64 == 0)
            bn /= 2;
        return bn;
    }

    // ---- kernels ---------------------------------------------------------

    // 128-channel layers run the pixels-on-N kernel (conv_pix.cu).
    bool use_pix() const { return precision != MG_PREC_FP32 && cpad == 128 && pix_mode != 0; }

    // Largest pixels per tile of the 128-channel kernel (its ranges are
    // balanced across SMs by the launcher).
    int choose_npx(int m_total) const {
        (void)m_total;
        return pix_npx > 0 ? pix_npx : 256;
    }

    // Whether the last trunk layer computes the head projection in its
    // epilogue (tensor-core path with one tile spanning all channels).
    // In the 16-bit modes the last trunk layer always computes the head
    // projection in its epilogue (one tile spans every channel); the fp32
    // verification mode runs it as a separate pass.
    bool fused_heads(int bucket) const {
        (void)bucket;
        return precision != MG_PREC_FP32;
    }

    // Buffers of layer li in the 16-bit modes, whose residual stream is the
    // pair (hi, lo): input conv stage -> (hi, lo); conv1 of a block hi -> t;
    // conv2 t + (hi, lo) -> (hi, lo) in place.  (The lo plane's layout is
    // the convolution kernel's own: 16-pixel blocks for the 128-channel
    // kernel, pixel-major for the other; all layers of a network use one.)
    void wire_hilo_layer(ConvLayer& L, int li, const void* stage, void* hi, uint16_t* lo,
                         void* t) const {
        if (li == 0) {
            L.in = stage;
            L.out16 = hi;
            L.out_lo = lo;
        } else if (li % 2 == 1) {
            L.in = hi;
            L.out16 = t;
        } else {
            L.in = t;
            L.res_hi = hi;
            L.res_lo = lo;
            L.out16 = hi;
            L.out_lo = lo;
        }
    }

    // The buffers a forward pass runs on: the engine's own (allocated for
    // max_batch positions) or a caller-provided set of the same roles.
    struct LayerBuffers {
        const void* stage;  // staged input rows
        float* x32;         // fp32 residual stream (the lo plane on the 16-bit paths)
        void* x16;          // 16-bit residual operand (hi plane)
        void* t;            // block-internal activation
        float* feat;        // head features
        int* err;           // device status word
    };
    LayerBuffers own_buffers() const { return {d_stage, d_x, d_x16, d_t, d_feat, d_err}; }

    ConvLayer layer_desc(int li, int bucket) const {
        return layer_desc(li, bucket * g.is, fused_heads(bucket), own_buffers());
    }

    // Layer li over m_total framed rows on buffer set b.
    ConvLayer layer_desc(int li, int m_total, bool fused, const LayerBuffers& b) const {
        ConvLayer L{};
        L.m_total = m_total;
        L.cin = wcin[li];
        L.cout = cpad;
        L.g = g;
        L.bias = d_bias[li];
        L.err = b.err;
        const bool f32 = precision == MG_PREC_FP32;
        L.weight = f32 ? (const void*)d_w32[li] : (const void*)d_w16[li];
        if (!f32) {
            wire_hilo_layer(L, li, b.stage, b.x16, reinterpret_cast<uint16_t*>(b.x32), b.t);
        } else if (li == 0) {  // input conv: staged planes -> x
            L.in = b.stage;
            L.out32 = b.x32;
        } else if (li % 2 == 1) {  // conv1 of a block: x -> t
            L.in = b.x32;
            L.out32 = reinterpret_cast<float*>(b.t);
        } else {  // conv2: t (+ x) -> x, in place over the residual rows
            L.in = b.t;
            L.res32 = b.x32;
            L.out32 = b.x32;
        }
        if (li == n_convs - 1 && fused) {
            // The trunk output is consumed only by the heads.
            L.out32 = nullptr;
            L.out16 = nullptr;
            L.out_lo = nullptr;
            L.head_w = d_head_w;
            L.head_b = d_head_b;
            L.feat = b.feat;
        }
        return L;
    }

    // One convolution layer as its own launch on `st`.
    void launch_layer(const ConvLayer& L, int li, cudaStream_t st) const {
        if (precision == MG_PREC_FP32) {
            ck(launch_conv_simt(L, st), "conv3x3_simt launch");
            return;
        }
        const bool fp16 = precision == MG_PREC_FP16;
        if (use_pix()) {
            ck(launch_conv_pix(L, choose_npx(L.m_total), fp16, num_sms, st), "conv3x3_pix launch");
            return;
        }
        // the head-projection layer's tile spans every channel
        const int bn = li == n_convs - 1 ? cpad : choose_bn(L.m_total);
        CUtensorMap ta, tb;
        const char* why = "";
        if (!make_conv_tensor_maps(L, bn, fp16, &ta, &tb, &why)) throw std::runtime_error(why);
        ck(launch_conv_tc(L, ta, tb, bn, fp16, num_sms, st), "conv3x3_tc launch");
    }

    void launch_conv(int li, int bucket) { launch_layer(layer_desc(li, bucket), li, stream); }

    // The 16-bit modes' limit on the network width (one tensor-core tile
    // spans every output channel of the head-projection layer).
    void check_width() const {
        if (precision != MG_PREC_FP32 && cpad > 256)
            throw std::runtime_error(
                "the bf16/fp16 modes support networks of up to 256 filters; use fp32");
    }

    // Whether the 128-channel trunk's CTAs own whole frames (frame stride of
    // whole 16-row chunks, one frame per tile at most).
    bool own_frames() const { return frame_trunk != 0 && g.is % 16 == 0 && g.is <= 256; }

    // Whether the 64/256-channel 16-bit trunk runs as persistent launches
    // (one tile spans every output channel).
    bool use_tc_trunk() const {
        return precision != MG_PREC_FP32 && !use_pix() && tc_trunk != 0 && n_convs > 1 && cpad <= 256;
    }

    // All trunk convolutions of a forward pass: persistent launches of the
    // 128-channel or the 64/256-channel tensor-core kernel, else one launch
    // per layer.
    void enqueue_trunk(int bucket) {
        if (use_pix() && pix_trunk) {
            std::vector<ConvLayer> layers(n_convs);
            for (int li = 0; li < n_convs; ++li) layers[li] = layer_desc(li, bucket);
            ck(launch_trunk_pix(layers.data(), n_convs, choose_npx(bucket * g.is),
                                precision == MG_PREC_FP16, num_sms, d_progress, stream,
                                withhold_cta, pix_trunk_min_tiles, own_frames()),
               "conv3x3_pix trunk launch");
        } else if (use_tc_trunk()) {
            std::vector<ConvLayer> layers(n_convs);
            for (int li = 0; li < n_convs; ++li) layers[li] = layer_desc(li, bucket);
            // Runs of at most trunk_tc_max_layers() layers; a run's first
            // layer takes its weights through its own tensor map.
            const int run = trunk_tc_max_layers();
            for (int l0 = 0; l0 < n_convs; l0 += run) {
                const int cnt = std::min(run, n_convs - l0);
                ck(launch_trunk_tc(layers.data() + l0, cnt, precision == MG_PREC_FP16, num_sms,
                                   d_progress, stream, withhold_cta),
                   "conv3x3_tc trunk launch");
            }
        } else {
            for (int li = 0; li < n_convs; ++li) launch_conv(li, bucket);
        }
    }

    int trunk_launches(int bucket) const {
        if (use_pix() && pix_trunk)
            return trunk_pix_launches(bucket * g.is, n_convs, choose_npx(bucket * g.is), num_sms,
                                      pix_trunk_min_tiles, own_frames());
        if (use_tc_trunk()) return (n_convs + trunk_tc_max_layers() - 1) / trunk_tc_max_layers();
        return n_convs;
    }

    void enqueue_trunk_heads(int bucket) {
        check_width();
        enqueue_trunk(bucket);
        if (!fused_heads(bucket))
            ck(launch_head_projection(d_x, bucket, cpad, g, d_head_w, d_head_b, d_feat, stream),
               "head projection launch");
        ck(launch_heads_fc(d_feat, fc, bucket, d_fc, d_probs, d_logits, d_value, stream),
           "heads launch");
    }

    void run_graph(int bucket) {
        if (!use_graphs) {
            enqueue_trunk_heads(bucket);
            return;
        }
        auto key = std::make_pair(bucket, precision);
        auto it = graphs.find(key);
        if (it == graphs.end()) {
            cudaGraph_t graph = nullptr;
            ck(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal),
               "cudaStreamBeginCapture");
            try {
                enqueue_trunk_heads(bucket);
            } catch (...) {
                cudaStreamEndCapture(stream, &graph);
                if (graph) cudaGraphDestroy(graph);
                throw;
            }
            ck(cudaStreamEndCapture(stream, &graph), "cudaStreamEndCapture");
            cudaGraphExec_t exec = nullptr;
            cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
            cudaGraphDestroy(graph);
            ck(e, "cudaGraphInstantiate");
            it = graphs.emplace(key, exec).first;
        }
        ck(cudaGraphLaunch(it->second, stream), "cudaGraphLaunch");
    }

    // Stage + trunk + heads for n <= max_batch positions at d_src (device).
    void forward_core(const float* d_src, int n) {
        const int bucket = bucket_for(n);
        ck(cudaMemsetAsync(d_err, 0, sizeof(int), stream), "cudaMemsetAsync(err)");
        ck(launch_stage_input(d_src, n, bucket, planes, g, kStagedChannels,
                              (flags & MG_FLAG_EIGEN_COMPAT) != 0, act_type(), d_stage, stream),
           "stage launch");
        run_graph(bucket);
        last_bucket = bucket;
    }

    // As forward_core for bit-packed inputs (device pointer).
    void forward_core_bits(const uint32_t* d_src, int n) {
        const int bucket = bucket_for(n);
        ck(cudaMemsetAsync(d_err, 0, sizeof(int), stream), "cudaMemsetAsync(err)");
        ck(launch_stage_bits(d_src, words_per_pos(), n, bucket, planes, g, kStagedChannels,
                             (flags & MG_FLAG_EIGEN_COMPAT) != 0, act_type(), d_stage, stream),
           "stage launch");
        run_graph(bucket);
        last_bucket = bucket;
    }

    // As forward_core for inputs in the history wire format (device pointer).
    void forward_core_history(const uint32_t* d_src, int n) {
        const int bucket = bucket_for(n);
        ck(cudaMemsetAsync(d_err, 0, sizeof(int), stream), "cudaMemsetAsync(err)");
        ck(launch_stage_history(d_src, history_words(), n, bucket, g, kStagedChannels,
                                (flags & MG_FLAG_EIGEN_COMPAT) != 0, act_type(), d_stage, stream),
           "stage launch");
        run_graph(bucket);
        last_bucket = bucket;
    }

    void check_ready() const {
        if (!loaded) throw std::logic_error("no model loaded");
    }
};

namespace {

int fail(mg_engine* e, int code, const std::string& msg) {
    if (e) e->err = msg;
    return code;
}

// Runs `fn` with the engine's device current, mapping exceptions to codes.
template <typename F>
int guarded(mg_engine* e, F&& fn) {
    if (e == nullptr) return MG_E_ARG;
    DeviceGuard dg(e->device);
    try {
        fn();
        e->err.clear();
        return MG_OK;
    } catch (const CudaFailure& f) {
        return fail(e, MG_E_CUDA, f.where + ": " + cudaGetErrorString(f.code));
    } catch (const std::invalid_argument& x) {
        return fail(e, MG_E_ARG, x.what());
    } catch (const std::logic_error& x) {
        return fail(e, MG_E_STATE, x.what());
    } catch (const std::runtime_error& x) {
        return fail(e, MG_E_MODEL, x.what());
    } catch (const std::exception& x) {
        return fail(e, MG_E_MODEL, x.what());
    }
}

bool is_pinned(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

}  // namespace

extern "C" {

mg_engine* mg_create(int device, int flags) {
    g_create_error.clear();
    int count = 0;
    cudaError_t ce = cudaGetDeviceCount(&count);
    if (ce != cudaSuccess || count == 0) {
        g_create_error = std::string("no CUDA device: ") + cudaGetErrorString(ce);
        cudaGetLastError();
        return nullptr;
    }
    if (device < 0 || device >= count) {
        g_create_error = "device index out of range";
        return nullptr;
    }
    std::unique_ptr<mg_engine> e(new mg_engine());
    e->device = device;
    e->flags = flags;
    DeviceGuard dg(device);
    cudaDeviceProp prop;
    if ((ce = cudaGetDeviceProperties(&prop, device)) != cudaSuccess) {
        g_create_error = std::string("cudaGetDeviceProperties: ") + cudaGetErrorString(ce);
        return nullptr;
    }
    if (prop.major != 10) {
        g_create_error = "this backend needs an sm_100 (B200-class) GPU; device " +
                         std::to_string(device) + " is sm_" + std::to_string(prop.major) +
                         std::to_string(prop.minor);
        return nullptr;
    }
    e->num_sms = prop.multiProcessorCount;
    if ((ce = cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking)) != cudaSuccess ||
        (ce = configure_conv_tc()) != cudaSuccess || (ce = configure_conv_pix()) != cudaSuccess) {
        g_create_error = std::string("CUDA setup failed: ") + cudaGetErrorString(ce);
        return nullptr;
    }
    if (const char* s = std::getenv("MG_CONV_BN")) e->conv_bn_override = std::atoi(s);
    if (const char* s = std::getenv("MG_NO_GRAPHS")) e->use_graphs = std::atoi(s) == 0;
    if (const char* s = std::getenv("MG_L2_POLICY")) e->l2_policy = std::atoi(s);
    if (const char* s = std::getenv("MG_PIX")) e->pix_mode = std::atoi(s);
    if (const char* s = std::getenv("MG_PIX_NPX")) e->pix_npx = std::atoi(s);
    if (const char* s = std::getenv("MG_PIX_TRUNK")) e->pix_trunk = std::atoi(s);
    if (const char* s = std::getenv("MG_TC_TRUNK")) e->tc_trunk = std::atoi(s);
    if (const char* s = std::getenv("MG_FRAME_TRUNK")) e->frame_trunk = std::atoi(s);
    if (const char* s = std::getenv("MG_PIX_TRUNK_MIN_TILES"))
        e->pix_trunk_min_tiles = std::max(1, std::atoi(s));
    if (const char* s = std::getenv("MG_TEST_WITHHOLD_PROGRESS")) e->withhold_cta = std::atoi(s);
    return e.release();
}

const char* mg_create_error(void) { return g_create_error.c_str(); }

void mg_destroy(mg_engine* e) { delete e; }

const char* mg_last_error(const mg_engine* e) { return e ? e->err.c_str() : "null engine"; }

int mg_load_onnx(mg_engine* e, const char* path) {
    if (path == nullptr) return fail(e, MG_E_ARG, "null path");
    return guarded(e, [&] {
        std::vector<NamedTensor> ts = read_onnx_initializers(path);
        std::vector<std::vector<float>> vals(ts.size());
        std::vector<TensorView> views(ts.size());
        for (size_t i = 0; i < ts.size(); ++i) {
            views[i].name = ts[i].name;
            views[i].dims = ts[i].dims;
            // Non-FLOAT tensors (e.g. num_batches_tracked) are kept without
            // values; reading one as a weight fails its size check.
            if (ts[i].data_type == 0 || ts[i].data_type == 1) vals[i] = ts[i].floats();
            views[i].data = vals[i].data();
            views[i].count = vals[i].size();
        }
        e->load(views);
    });
}

int mg_load_weights(mg_engine* e, const mg_tensor* tensors, int count) {
    if (count < 0 || (count > 0 && tensors == nullptr)) return fail(e, MG_E_ARG, "bad tensor list");
    return guarded(e, [&] {
        std::vector<TensorView> views(count);
        for (int i = 0; i < count; ++i) {
            const mg_tensor& t = tensors[i];
            if (t.name == nullptr || t.ndims < 0 || (t.ndims > 0 && t.dims == nullptr))
                throw std::invalid_argument("tensor " + std::to_string(i) + " is malformed");
            views[i].name = t.name;
            views[i].dims.assign(t.dims, t.dims + t.ndims);
            size_t cnt = t.ndims > 0 ? 1 : 0;
            for (int d = 0; d < t.ndims; ++d) cnt *= (size_t)std::max<int64_t>(t.dims[d], 0);
            views[i].data = t.data;
            views[i].count = t.data ? cnt : 0;
        }
        e->load(views);
    });
}

int mg_get_info(const mg_engine* e, int* board_size, int* input_channels, int* num_filters,
                int* num_res_blocks, int* action_size) {
    if (e == nullptr) return MG_E_ARG;
    if (!e->loaded) return MG_E_STATE;
    if (board_size) *board_size = e->net.board;
    if (input_channels) *input_channels = e->net.input_channels;
    if (num_filters) *num_filters = e->net.filters;
    if (num_res_blocks) *num_res_blocks = e->net.blocks;
    if (action_size) *action_size = e->net.actions;
    return MG_OK;
}

int mg_set_precision(mg_engine* e, int precision) {
    if (e == nullptr) return MG_E_ARG;
    if (precision != MG_PREC_BF16 && precision != MG_PREC_FP16 && precision != MG_PREC_FP32)
        return fail(e, MG_E_ARG, "unknown precision");
    return guarded(e, [&] {
        e->precision = precision;
        if (e->loaded) e->prepare_weights();
    });
}

int mg_set_max_batch(mg_engine* e, int max_batch) {
    if (e == nullptr) return MG_E_ARG;
    if (max_batch < 1 || max_batch > 65536) return fail(e, MG_E_ARG, "max batch out of range");
    return guarded(e, [&] {
        e->max_batch = max_batch;
        e->free_buffers();
    });
}

int mg_forward(mg_engine* e, const float* states, int n, float* policy_out, float* value_out,
               float* logits_out) {
    if (e == nullptr) return MG_E_ARG;
    if (n < 0) return fail(e, MG_E_ARG, "negative batch size");
    if (n == 0) return MG_OK;
    if (states == nullptr || policy_out == nullptr || value_out == nullptr)
        return fail(e, MG_E_ARG, "null buffer");
    int dev_err = 0;
    int rc = guarded(e, [&] {
        e->check_ready();
        e->prepare_weights();
        e->ensure_buffers();
        const size_t in_per = (size_t)e->planes * e->hw;
        const int A = e->actions;
        const bool pinned = is_pinned(states);
        for (int base = 0; base < n; base += e->max_batch) {
            const int m = std::min(e->max_batch, n - base);
            const float* src = states + (size_t)base * in_per;
            if (pinned) {
                ck(cudaMemcpyAsync(e->d_states, src, (size_t)m * in_per * sizeof(float),
                                   cudaMemcpyHostToDevice, e->stream),
                   "cudaMemcpyAsync(H2D states)");
            } else {
                // The pinned staging buffer may still feed the previous chunk's copy.
                ck(cudaStreamSynchronize(e->stream), "cudaStreamSynchronize");
                std::memcpy(e->h_states, src, (size_t)m * in_per * sizeof(float));
                ck(cudaMemcpyAsync(e->d_states, e->h_states, (size_t)m * in_per * sizeof(float),
                                   cudaMemcpyHostToDevice, e->stream),
                   "cudaMemcpyAsync(H2D states)");
            }
            e->forward_core(e->d_states, m);
            ck(cudaMemcpyAsync(policy_out + (size_t)base * A, e->d_probs, (size_t)m * A * sizeof(float),
                               cudaMemcpyDeviceToHost, e->stream),
               "cudaMemcpyAsync(D2H policy)");
            ck(cudaMemcpyAsync(value_out + base, e->d_value, (size_t)m * sizeof(float),
                               cudaMemcpyDeviceToHost, e->stream),
               "cudaMemcpyAsync(D2H value)");
            if (logits_out)
                ck(cudaMemcpyAsync(logits_out + (size_t)base * A, e->d_logits,
                                   (size_t)m * A * sizeof(float), cudaMemcpyDeviceToHost, e->stream),
                   "cudaMemcpyAsync(D2H logits)");
            ck(cudaMemcpyAsync(e->h_err, e->d_err, sizeof(int), cudaMemcpyDeviceToHost, e->stream),
               "cudaMemcpyAsync(D2H status)");
            if (base + m < n) {
                // Later chunks reuse the device buffers: keep results ordered.
                ck(cudaStreamSynchronize(e->stream), "cudaStreamSynchronize");
                dev_err |= *e->h_err;
            }
        }
        ck(cudaStreamSynchronize(e->stream), "cudaStreamSynchronize");
        dev_err |= *e->h_err;
    });
    if (rc == MG_OK && dev_err != 0)
        return fail(e, MG_E_DEVICE, "a kernel gave up waiting (device status " +
                                        std::to_string(dev_err) + ")");
    return rc;
}

int mg_forward_device(mg_engine* e, const float* d_states, int n, float* d_policy, float* d_value,
                      float* d_logits) {
    if (e == nullptr) return MG_E_ARG;
    if (n < 0) return fail(e, MG_E_ARG, "negative batch size");
    if (n == 0) return MG_OK;
    if (d_states == nullptr || d_policy == nullptr || d_value == nullptr)
        return fail(e, MG_E_ARG, "null buffer");
    if (n > e->max_batch) return fail(e, MG_E_ARG, "batch exceeds the max batch");
    return guarded(e, [&] {
        e->check_ready();
        e->prepare_weights();
        e->ensure_buffers();
        const int A = e->actions;
        e->forward_core(d_states, n);
        ck(cudaMemcpyAsync(d_policy, e->d_probs, (size_t)n * A * sizeof(float),
                           cudaMemcpyDeviceToDevice, e->stream),
           "cudaMemcpyAsync(policy)");
        ck(cudaMemcpyAsync(d_value, e->d_value, (size_t)n * sizeof(float), cudaMemcpyDeviceToDevice,
                           e->stream),
           "cudaMemcpyAsync(value)");
        if (d_logits)
            ck(cudaMemcpyAsync(d_logits, e->d_logits, (size_t)n * A * sizeof(float),
                               cudaMemcpyDeviceToDevice, e->stream),
               "cudaMemcpyAsync(logits)");
    });
}

int mg_words_per_position(const mg_engine* e) {
    if (e == nullptr || !e->loaded) return 0;
    return e->words_per_pos();
}

int mg_pack_states(const float* states, int n, int state_size, uint32_t* out) {
    if (n < 0 || state_size <= 0 || (n > 0 && (states == nullptr || out == nullptr))) return MG_E_ARG;
    const int words = (state_size + 31) / 32;
    for (int i = 0; i < n; ++i) {
        const float* s = states + (size_t)i * state_size;
        uint32_t* w = out + (size_t)i * words;
        for (int k = 0; k < words; ++k) {
            uint32_t v = 0;
            const int lo = k * 32, hi = std::min(state_size, lo + 32);
            for (int j = lo; j < hi; ++j) {
                const float x = s[j];
                if (x == 1.0f) v |= 1u << (j - lo);
                else if (x != 0.0f) return MG_E_ARG;  // not a binary plane
            }
            w[k] = v;
        }
    }
    return MG_OK;
}

}  // extern "C"

namespace {

// Host-buffer forward of n positions of `words` 32-bit words each (one of
// the packed wire formats): chunks of up to max_batch positions are copied
// into the engine's device buffer e->*d_buf (straight from the caller's
// buffer when it is page-locked, else through the pinned e->*h_buf), staged
// by (e->*core)(device pointer, count), and the results copied back.
int forward_words(mg_engine* e, const uint32_t* src_all, int n, float* policy_out,
                  float* value_out, float* logits_out, int (mg_engine::*words_fn)() const,
                  uint32_t* mg_engine::*d_buf, uint32_t* mg_engine::*h_buf,
                  void (mg_engine::*core)(const uint32_t*, int)) {
    if (e == nullptr) return MG_E_ARG;
    if (n < 0) return fail(e, MG_E_ARG, "negative batch size");
    if (n == 0) return MG_OK;
    if (src_all == nullptr || policy_out == nullptr || value_out == nullptr)
        return fail(e, MG_E_ARG, "null buffer");
    int dev_err = 0;
    int rc = guarded(e, [&] {
        e->check_ready();
        e->prepare_weights();
        e->ensure_buffers();
        const size_t words = (size_t)(e->*words_fn)();
        const int A = e->actions;
        const bool pinned = is_pinned(src_all);
        for (int base = 0; base < n; base += e->max_batch) {
            const int m = std::min(e->max_batch, n - base);
            const uint32_t* src = src_all + (size_t)base * words;
            if (pinned) {
                ck(cudaMemcpyAsync(e->*d_buf, src, (size_t)m * words * 4, cudaMemcpyHostToDevice,
                                   e->stream),
                   "cudaMemcpyAsync(H2D inputs)");
            } else {
                ck(cudaStreamSynchronize(e->stream), "cudaStreamSynchronize");
                std::memcpy(e->*h_buf, src, (size_t)m * words * 4);
                ck(cudaMemcpyAsync(e->*d_buf, e->*h_buf, (size_t)m * words * 4,
                                   cudaMemcpyHostToDevice, e->stream),
                   "cudaMemcpyAsync(H2D inputs)");
            }
            (e->*core)(e->*d_buf, m);
            ck(cudaMemcpyAsync(policy_out + (size_t)base * A, e->d_probs, (size_t)m * A * sizeof(float),
                               cudaMemcpyDeviceToHost, e->stream),
               "cudaMemcpyAsync(D2H policy)");
            ck(cudaMemcpyAsync(value_out + base, e->d_value, (size_t)m * sizeof(float),
                               cudaMemcpyDeviceToHost, e->stream),
               "cudaMemcpyAsync(D2H value)");
            if (logits_out)
                ck(cudaMemcpyAsync(logits_out + (size_t)base * A, e->d_logits,
                                   (size_t)m * A * sizeof(float), cudaMemcpyDeviceToHost, e->stream),
                   "cudaMemcpyAsync(D2H logits)");
            ck(cudaMemcpyAsync(e->h_err, e->d_err, sizeof(int), cudaMemcpyDeviceToHost, e->stream),
               "cudaMemcpyAsync(D2H status)");
            if (base + m < n) {
                ck(cudaStreamSynchronize(e->stream), "cudaStreamSynchronize");
                dev_err |= *e->h_err;
            }
        }
        ck(cudaStreamSynchronize(e->stream), "cudaStreamSynchronize");
        dev_err |= *e->h_err;
    });
    if (rc == MG_OK && dev_err != 0)
        return fail(e, MG_E_DEVICE, "a kernel gave up waiting (device status " +
                                        std::to_string(dev_err) + ")");
    return rc;
}

}  // namespace

extern "C" {

int mg_forward_packed(mg_engine* e, const uint32_t* bits, int n, float* policy_out,
                      float* value_out, float* logits_out) {
    return forward_words(e, bits, n, policy_out, value_out, logits_out, &mg_engine::words_per_pos,
                         &mg_engine::d_bits, &mg_engine::h_bits, &mg_engine::forward_core_bits);
}

int mg_submit_packed(mg_engine* e, const uint32_t* bits, int n, float* policy_out, float* value_out,
                     int* ticket) {
    if (e == nullptr) return MG_E_ARG;
    if (ticket == nullptr || bits == nullptr || policy_out == nullptr || value_out == nullptr)
        return fail(e, MG_E_ARG, "null buffer");
    if (n < 1 || n > e->max_batch) return fail(e, MG_E_ARG, "batch size out of range");
    if (!is_pinned(bits) || !is_pinned(policy_out) || !is_pinned(value_out))
        return fail(e, MG_E_ARG, "mg_submit_packed needs page-locked input and output buffers");
    return guarded(e, [&] {
        e->check_ready();
        e->prepare_weights();
        e->ensure_buffers();
        const int slot = e->next_ticket % mg_engine::kTickets;
        if (e->tick_ev[slot] == nullptr)
            ck(cudaEventCreateWithFlags(&e->tick_ev[slot], cudaEventDisableTiming), "cudaEventCreate");
        // A ticket slot is reused kTickets submissions later: the caller has
        // waited for that one long since (at most two are outstanding).
        ck(cudaEventSynchronize(e->tick_ev[slot]), "cudaEventSynchronize");
        const size_t words = (size_t)e->words_per_pos();
        const int A = e->actions;
        ck(cudaMemcpyAsync(e->d_bits, bits, (size_t)n * words * 4, cudaMemcpyHostToDevice, e->stream),
           "cudaMemcpyAsync(H2D bits)");
        e->forward_core_bits(e->d_bits, n);
        ck(cudaMemcpyAsync(policy_out, e->d_probs, (size_t)n * A * sizeof(float), cudaMemcpyDeviceToHost,
                           e->stream),
           "cudaMemcpyAsync(D2H policy)");
        ck(cudaMemcpyAsync(value_out, e->d_value, (size_t)n * sizeof(float), cudaMemcpyDeviceToHost,
                           e->stream),
           "cudaMemcpyAsync(D2H value)");
        ck(cudaMemcpyAsync(e->h_tick_err + slot, e->d_err, sizeof(int), cudaMemcpyDeviceToHost,
                           e->stream),
           "cudaMemcpyAsync(D2H status)");
        ck(cudaEventRecord(e->tick_ev[slot], e->stream), "cudaEventRecord");
        *ticket = e->next_ticket.fetch_add(1);
    });
}

int mg_wait_submitted(mg_engine* e, int ticket) {
    // Touches only the ticket's event and status word (not the engine's
    // error message), so one thread may wait while another submits.
    const int issued = e != nullptr ? e->next_ticket.load() : 0;
    if (e == nullptr || ticket < 0 || ticket >= issued || ticket < issued - mg_engine::kTickets)
        return MG_E_ARG;
    const int slot = ticket % mg_engine::kTickets;
    DeviceGuard dg(e->device);
    if (cudaEventSynchronize(e->tick_ev[slot]) != cudaSuccess) {
        cudaGetLastError();
        return MG_E_CUDA;
    }
    return e->h_tick_err[slot] != 0 ? MG_E_DEVICE : MG_OK;
}

int mg_history_words(const mg_engine* e) {
    if (e == nullptr || !e->loaded) return 0;
    return e->history_words();
}

int mg_forward_history(mg_engine* e, const uint32_t* history, int n, float* policy_out,
                       float* value_out, float* logits_out) {
    if (e != nullptr && e->loaded && e->planes != 2 * kHistoryBoards + 1)
        return fail(e, MG_E_ARG, "the history wire format needs a network of 17 input planes");
    return forward_words(e, history, n, policy_out, value_out, logits_out,
                         &mg_engine::history_words, &mg_engine::d_hist, &mg_engine::h_hist,
                         &mg_engine::forward_core_history);
}

int mg_synchronize(mg_engine* e) {
    if (e == nullptr) return MG_E_ARG;
    int dev_err = 0;
    int rc = guarded(e, [&] {
        ck(cudaStreamSynchronize(e->stream), "cudaStreamSynchronize");
        if (e->d_err) {
            ck(cudaMemcpy(&dev_err, e->d_err, sizeof(int), cudaMemcpyDeviceToHost),
               "cudaMemcpy(status)");
        }
    });
    if (rc == MG_OK && dev_err != 0)
        return fail(e, MG_E_DEVICE, "a kernel gave up waiting (device status " +
                                        std::to_string(dev_err) + ")");
    return rc;
}

void* mg_stream(mg_engine* e) { return e ? (void*)e->stream : nullptr; }

float* mg_host_input(mg_engine* e) {
    if (e == nullptr) return nullptr;
    float* out = nullptr;
    guarded(e, [&] {
        e->check_ready();
        e->ensure_buffers();
        out = e->h_states;
    });
    return out;
}

uint32_t* mg_host_bits(mg_engine* e) {
    if (e == nullptr) return nullptr;
    uint32_t* out = nullptr;
    guarded(e, [&] {
        e->check_ready();
        e->ensure_buffers();
        out = e->h_bits;
    });
    return out;
}

void* mg_host_alloc(size_t bytes) {
    void* p = nullptr;
    if (bytes == 0 || cudaMallocHost(&p, bytes) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return p;
}

void mg_host_free(void* p) {
    if (p != nullptr) cudaFreeHost(p);
}

int mg_max_batch(const mg_engine* e) { return e ? e->max_batch : 0; }

int mg_launch_conv(mg_engine* e, int n, int layer, int reps) {
    if (e == nullptr) return MG_E_ARG;
    return guarded(e, [&] {
        e->check_ready();
        if (e->last_bucket == 0 || e->alloc_batch == 0)
            throw std::logic_error("run a forward pass before mg_launch_conv");
        if (layer < 0 || layer >= 2 * e->net.blocks || reps < 0 || n < 1 || n > e->max_batch)
            throw std::invalid_argument("bad layer, n or reps");
        const int bucket = e->bucket_for(n);
        for (int r = 0; r < reps; ++r) e->launch_conv(1 + layer, bucket);
    });
}

int mg_launch_trunk(mg_engine* e, int n, int reps) {
    if (e == nullptr) return MG_E_ARG;
    return guarded(e, [&] {
        e->check_ready();
        if (e->last_bucket == 0 || e->alloc_batch == 0)
            throw std::logic_error("run a forward pass before mg_launch_trunk");
        if (reps < 0 || n < 1 || n > e->max_batch) throw std::invalid_argument("bad n or reps");
        const int bucket = e->bucket_for(n);
        for (int r = 0; r < reps; ++r) e->enqueue_trunk(bucket);
    });
}

int mg_launches_per_forward(mg_engine* e, int n) {
    if (e == nullptr || !e->loaded) return 0;
    const int bucket = e->bucket_for(std::max(1, std::min(n, e->max_batch)));
    return 1 /* stage */ + e->trunk_launches(bucket) + (e->fused_heads(bucket) ? 0 : 1) +
           2 /* FC, finish */;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Forward pass that allocates nothing.
//
// mg_forward_device allocates its activation buffers on an engine's first
// forward (and again after mg_set_max_batch).  Some callers cannot let a
// library call cudaMalloc once they are running: cudaMalloc and especially
// cudaFree synchronise the whole device, stalling every other stream the
// process has in flight, and a host program that reserves all of its GPU
// memory up front (or runs under a fixed memory budget) must not see an
// allocation fail in the middle of a search.  For them this variant takes
// every intermediate buffer - staged input, fp32 residual stream, 16-bit
// operands, head features, FC outputs and the status word - from one
// file-scope __device__ arena of kNoAllocArenaBytes, which each GPU that
// loads this library holds until the process exits.
//
// The arena's device address is looked up once per device with
// cudaGetSymbolAddress on the first call made on that device (so make that
// first call before any stream capture); in host code the array's name is
// only a host-side stand-in and must never be handed to a kernel.  All calls
// on a device share the one arena, which keeps whatever the previous call
// left there: every buffer is fully rewritten by each call except the
// status word, which is cleared first.  Calls whose work overlaps on the GPU
// (two engines on the same device, or two streams) race on the arena and
// must be serialised by the caller.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kNoAllocArenaBytes = size_t(32) << 20;  // 32 MiB per device
__device__ __align__(256) unsigned char g_noalloc_arena[kNoAllocArenaBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};

// Device address of the arena for `dev` (which must be current).
cudaError_t noalloc_arena(int dev, void** out) {
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_ptr[dev] == nullptr) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_arena);
        if (e != cudaSuccess) return e;
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return cudaSuccess;
}

// Carves the per-call buffers for n positions out of the arena; returns the
// bytes needed (which may exceed the arena, in which case nothing is set).
struct NoAllocBuffers {
    void* stage;
    float* x32;  // fp32 residual stream (its fp16 remainder plane on the 128-channel path)
    void* x16;
    void* t;
    float* feat;
    float* fc;
    float* logits;
    int* err;
};

size_t noalloc_layout(const mg_engine* e, int n, unsigned char* base, NoAllocBuffers* b) {
    const size_t rows = (size_t)n * e->g.is;
    const size_t elem = e->elem_bytes();
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off += (bytes + 255) / 256 * 256;
        return at;
    };
    const size_t o_stage = take(rows * kStagedChannels * elem);
    const size_t o_x32 = take(rows * e->cpad * 4);
    const size_t o_x16 = take(rows * e->cpad * 2);
    const size_t o_t = take(rows * e->cpad * elem);
    const size_t o_feat = take((size_t)n * 3 * e->hw * 4);
    const size_t o_fc = take((size_t)kHeadsFcSplits * n * (e->actions + e->net.hidden) * 4);
    const size_t o_log = take((size_t)n * e->actions * 4);
    const size_t o_err = take(sizeof(int));
    if (base != nullptr && off <= kNoAllocArenaBytes) {
        b->stage = base + o_stage;
        b->x32 = reinterpret_cast<float*>(base + o_x32);
        b->x16 = base + o_x16;
        b->t = base + o_t;
        b->feat = reinterpret_cast<float*>(base + o_feat);
        b->fc = reinterpret_cast<float*>(base + o_fc);
        b->logits = reinterpret_cast<float*>(base + o_log);
        b->err = reinterpret_cast<int*>(base + o_err);
    }
    return off;
}

}  // namespace

extern "C" int mg_forward_device_noalloc(mg_engine* e, const float* d_states, int n,
                                         float* d_policy, float* d_value, float* d_logits) {
    if (e == nullptr) return MG_E_ARG;
    if (n < 0) return fail(e, MG_E_ARG, "negative batch size");
    if (n == 0) return MG_OK;
    if (d_states == nullptr || d_policy == nullptr || d_value == nullptr)
        return fail(e, MG_E_ARG, "null buffer");
    int dev_err = 0;
    int rc = guarded(e, [&] {
        e->check_ready();
        const bool f32 = e->precision == MG_PREC_FP32;
        if (f32 ? e->d_w32.size() != (size_t)e->n_convs : e->w16_prec != e->precision)
            throw std::logic_error("weights for the current precision are not on the device");
        e->check_width();  // before anything is enqueued
        // Largest batch that fits the arena, for the error message.
        int cap = 0;
        while (noalloc_layout(e, cap + 1, nullptr, nullptr) <= kNoAllocArenaBytes) ++cap;
        if (n > cap)
            throw std::invalid_argument("batch of " + std::to_string(n) +
                                        " positions exceeds the no-allocation scratch arena (" +
                                        std::to_string(kNoAllocArenaBytes >> 20) +
                                        " MiB): at most " + std::to_string(cap) +
                                        " positions for this network");
        void* arena = nullptr;
        ck(noalloc_arena(e->device, &arena), "cudaGetSymbolAddress(no-allocation arena)");
        NoAllocBuffers b{};
        noalloc_layout(e, n, reinterpret_cast<unsigned char*>(arena), &b);
        cudaStream_t st = e->stream;
        ck(cudaMemsetAsync(b.err, 0, sizeof(int), st), "cudaMemsetAsync(status)");
        ck(launch_stage_input(d_states, n, n, e->planes, e->g, kStagedChannels,
                              (e->flags & MG_FLAG_EIGEN_COMPAT) != 0, e->act_type(), b.stage, st),
           "stage launch");
        const bool fused = e->fused_heads(n);
        const mg_engine::LayerBuffers lb{b.stage, b.x32, b.x16, b.t, b.feat, b.err};
        for (int li = 0; li < e->n_convs; ++li)
            e->launch_layer(e->layer_desc(li, n * e->g.is, fused, lb), li, st);
        if (!fused)
            ck(launch_head_projection(b.x32, n, e->cpad, e->g, e->d_head_w, e->d_head_b, b.feat, st),
               "head projection launch");
        ck(launch_heads_fc(b.feat, e->fc, n, b.fc, d_policy, d_logits ? d_logits : b.logits, d_value,
                           st),
           "heads launch");
        ck(cudaMemcpyAsync(&dev_err, b.err, sizeof(int), cudaMemcpyDeviceToHost, st),
           "cudaMemcpyAsync(status)");
        ck(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    });
    if (rc == MG_OK && dev_err != 0)
        return fail(e, MG_E_DEVICE, "a kernel gave up waiting (device status " +
                                        std::to_string(dev_err) + ")");
    return rc;
}


