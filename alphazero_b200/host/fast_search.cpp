#include "fast_search.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <exception>
#include <new>
#include <numeric>
#include <stdexcept>
#include <type_traits>

namespace mgb {

namespace {
enum : int { kUnevaluated = 0, kExpanding = 1, kExpanded = 2 };
}

struct FastSearch::Node {
    std::atomic<int> visits{0};
    std::atomic<int> vloss{0};
    std::atomic<int> state{kUnevaluated};
    std::atomic<int32_t> value_bits{0};  // float total value
    float prior = 0.0f;
    int action = -1;
    Node* children = nullptr;  // n_children nodes, legal actions ascending (arena memory)
    int n_children = 0;

    // The total value as a float updated by compare-and-swap
    // (include/mcts.h:38-55).
    void add_value(float v) {
        int32_t old_bits = value_bits.load(std::memory_order_relaxed);
        int32_t new_bits;
        float old_f, new_f;
        do {
            std::memcpy(&old_f, &old_bits, sizeof(float));
            new_f = old_f + v;
            std::memcpy(&new_bits, &new_f, sizeof(float));
        } while (!value_bits.compare_exchange_weak(old_bits, new_bits, std::memory_order_relaxed));
    }
    float total_value() const {
        const int32_t bits = value_bits.load(std::memory_order_relaxed);
        float f;
        std::memcpy(&f, &bits, sizeof(float));
        return f;
    }
};

namespace {
constexpr size_t kArenaBlockBytes = size_t(256) << 10;
}

// n default-constructed nodes from the arena (a fresh block when the
// current one is full; blocks hold at least one 362-child array).
FastSearch::Node* FastSearch::Arena::take(int n) {
    const size_t bytes = (size_t)n * sizeof(Node);
    if (block < blocks.size() && used + bytes > kArenaBlockBytes) {
        ++block;
        used = 0;
    }
    if (block == blocks.size()) blocks.emplace_back(new unsigned char[kArenaBlockBytes]);
    Node* out = reinterpret_cast<Node*>(blocks[block].get() + used);
    used += (bytes + alignof(Node) - 1) / alignof(Node) * alignof(Node);
    for (int i = 0; i < n; ++i) new (&out[i]) Node();
    return out;
}

FastSearch::FastSearch(PackedEvaluator* evaluator, int board_size, const SearchParams& params,
                       uint64_t seed)
    : evaluator_(evaluator),
      board_(board_size),
      actions_(board_size * board_size + 1),
      words_((kInputPlanes * board_size * board_size + 31) / 32),
      params_(params),
      rng_((std::mt19937::result_type)seed) {
    if (evaluator_ == nullptr || board_size < 2 || board_size > kMaxBoard || params_.simulations < 1)
        throw std::invalid_argument("FastSearch: bad arguments");
    static_assert(std::is_trivially_destructible<Node>::value, "arena nodes are never destroyed");
    if ((size_t)actions_ * sizeof(Node) > kArenaBlockBytes)
        throw std::invalid_argument("FastSearch: arena block too small");
    const int extra = params_.grouped ? 0 : std::max(1, params_.threads) - 1;
    arenas_.resize(extra + 1);
    if (params_.grouped) {
        const int t = std::max(1, params_.threads);
        group_.paths.resize(t);
        for (auto& p : group_.paths) p.reserve(64);
        group_.leaves.resize(t);
        group_.words.resize((size_t)t * words_);
        group_.policy.resize((size_t)t * actions_);
        group_.values.resize(t);
        group_.legal.resize((size_t)t * actions_);
        group_.word_ptrs.resize(t);
        group_.policy_ptrs.resize(t);
        for (int i = 0; i < t; ++i) {
            group_.word_ptrs[i] = group_.words.data() + (size_t)i * words_;
            group_.policy_ptrs[i] = group_.policy.data() + (size_t)i * actions_;
        }
    }
    for (int i = 0; i < extra; ++i) pool_.emplace_back(&FastSearch::worker_loop, this, i + 1);
}

FastSearch::~FastSearch() {
    {
        std::lock_guard<std::mutex> lock(mu_);
        stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : pool_) t.join();
}

// MCTSNode::select_child / ucb_score / q_value (src/mcts.cpp:13-25,
// include/mcts.h:57-78): the same expressions; sqrt(parent total) once.
FastSearch::Node* FastSearch::select_child(Node* node) const {
    const int parent_total =
        node->visits.load(std::memory_order_relaxed) + node->vloss.load(std::memory_order_relaxed);
    const float sq = std::sqrt((float)parent_total);
    Node* best = nullptr;
    float best_score = -1e9f;
    for (int i = 0; i < node->n_children; ++i) {
        Node& c = node->children[i];
        const int vc = c.visits.load(std::memory_order_relaxed);
        const int vl = c.vloss.load(std::memory_order_relaxed);
        const int total = vc + vl;
        const float q = total == 0 ? 0.0f : (c.total_value() - (float)vl) / (float)total;
        const float u = params_.c_puct * c.prior * sq / (1.0f + total);
        const float score = q + u;
        if (score > best_score) {
            best_score = score;
            best = &c;
        }
    }
    return best;
}

// MCTS::mask_policy + MCTS::expand (src/mcts.cpp:43-73).
void FastSearch::expand(Node* node, float* policy, const uint8_t* legal, Arena& arena) {
    float sum = 0.0f;
    int k = 0;
    for (int a = 0; a < actions_; ++a) {
        policy[a] *= (float)legal[a];
        sum += policy[a];
        k += legal[a] != 0;
    }
    if (sum > 0.0f) {
        for (int a = 0; a < actions_; ++a) policy[a] /= sum;
    } else {
        float ls = 0.0f;
        for (int a = 0; a < actions_; ++a) ls += (float)legal[a];
        for (int a = 0; a < actions_; ++a) policy[a] = (float)legal[a] / ls;
    }
    Node* kids = arena.take(k);
    for (int a = 0, i = 0; a < actions_; ++a) {
        if (!legal[a]) continue;
        kids[i].action = a;
        kids[i].prior = policy[a];
        ++i;
    }
    node->children = kids;
    node->n_children = k;
}

// MCTS::backprop (src/mcts.cpp:85-94).
void FastSearch::backup(std::vector<Node*>& path, float value) {
    float v = value;
    for (int i = (int)path.size() - 1; i >= 0; --i) {
        Node* n = path[i];
        n->vloss.fetch_sub(1, std::memory_order_relaxed);
        n->visits.fetch_add(1, std::memory_order_relaxed);
        n->add_value(v);
        v = -v;
    }
}

// MCTS::revert_virtual_losses (src/mcts.cpp:101-104).
void FastSearch::revert(std::vector<Node*>& path) {
    for (Node* n : path) n->vloss.fetch_sub(1, std::memory_order_relaxed);
}

// MCTS::dirichlet + add_dirichlet_noise (src/mcts.cpp:31-41, :75-83).
void FastSearch::add_dirichlet_noise(Node* root) {
    std::gamma_distribution<float> gamma(params_.dirichlet_alpha, 1.0f);
    std::vector<float> noise(actions_);
    float sum = 0.0f;
    for (int a = 0; a < actions_; ++a) {
        noise[a] = gamma(rng_);
        sum += noise[a];
    }
    if (sum > 0.0f)
        for (auto& x : noise) x /= sum;
    const float eps = params_.dirichlet_epsilon;
    for (int i = 0; i < root->n_children; ++i) {
        Node& c = root->children[i];
        c.prior = (1.0f - eps) * c.prior + eps * noise[c.action];
    }
}

// MCTS::search_thread_loop (src/mcts.cpp:126-165) for one search thread.
void FastSearch::playouts_from_root(int tid) {
    Arena& arena = arenas_[tid];
    std::vector<Node*> path;
    path.reserve(64);
    std::vector<uint32_t> words(words_);
    std::vector<float> policy(actions_);
    std::vector<uint8_t> legal(actions_);
    const int target = params_.simulations;
    try {
        while (sims_done_.load(std::memory_order_relaxed) < target) {
            Node* node = root_;
            GoPosition g = *pos_;
            path.clear();
            path.push_back(node);
            node->vloss.fetch_add(1, std::memory_order_relaxed);
            bool collision = false;
            for (;;) {
                const int st = node->state.load(std::memory_order_acquire);
                if (st == kExpanded) {
                    Node* child = select_child(node);
                    if (child == nullptr) break;
                    child->vloss.fetch_add(1, std::memory_order_relaxed);
                    path.push_back(child);
                    g.play(child->action);
                    node = child;
                } else if (st == kExpanding) {
                    collision = true;  // another thread is evaluating it
                    break;
                } else {
                    break;  // an unevaluated leaf
                }
            }
            if (collision) {
                revert(path);
                std::this_thread::yield();
                continue;
            }
            if (g.over()) {
                const float v = g.winner() == 0 ? 0.0f : (g.winner() == g.to_move() ? 1.0f : -1.0f);
                backup(path, v);
                sims_done_.fetch_add(1, std::memory_order_relaxed);
                playouts_.fetch_add(1, std::memory_order_relaxed);
                continue;
            }
            int expected = kUnevaluated;
            if (!node->state.compare_exchange_strong(expected, kExpanding, std::memory_order_acq_rel)) {
                revert(path);
                std::this_thread::yield();
                continue;
            }
            float value = 0.0f;
            g.encode_bits(words.data());
            evaluator_->evaluate_packed(words.data(), words_, policy.data(), &value);
            g.legal_mask(legal.data());
            expand(node, policy.data(), legal.data(), arena);
            node->state.store(kExpanded, std::memory_order_release);
            backup(path, value);
            sims_done_.fetch_add(1, std::memory_order_relaxed);
            playouts_.fetch_add(1, std::memory_order_relaxed);
        }
    } catch (...) {
        // End every thread's loop (a node left EXPANDING would make the
        // others retry forever) and hand the error to search().
        sims_done_.store(target, std::memory_order_relaxed);
        std::lock_guard<std::mutex> lock(mu_);
        if (!error_) error_ = std::current_exception();
    }
}

// The params.threads concurrent playouts of MCTS::search as rounds on the
// calling thread (SearchParams::grouped): the descent, collision rule,
// terminal valuation, masking, expansion and backup of playouts_from_root,
// with the leaves of a round evaluated as one group.
void FastSearch::grouped_playouts() {
    const int t = std::max(1, params_.threads);
    const int target = params_.simulations;
    Arena& arena = arenas_[0];
    int done = 0;
    while (done < target) {
        int n = 0;
        const int want = std::min(t, target - done);
        while (n < want && done < target) {
            std::vector<Node*>& path = group_.paths[n];
            Node* node = root_;
            GoPosition g = *pos_;
            path.clear();
            path.push_back(node);
            node->vloss.fetch_add(1, std::memory_order_relaxed);
            bool collision = false;
            for (;;) {
                const int st = node->state.load(std::memory_order_relaxed);
                if (st == kExpanded) {
                    Node* child = select_child(node);
                    if (child == nullptr) break;
                    child->vloss.fetch_add(1, std::memory_order_relaxed);
                    path.push_back(child);
                    g.play(child->action);
                    node = child;
                } else if (st == kExpanding) {
                    collision = true;  // already a leaf of this round
                    break;
                } else {
                    break;  // an unevaluated leaf
                }
            }
            if (collision) {
                revert(path);
                break;  // the round is complete
            }
            if (g.over()) {
                const float v = g.winner() == 0 ? 0.0f : (g.winner() == g.to_move() ? 1.0f : -1.0f);
                backup(path, v);
                ++done;
                playouts_.fetch_add(1, std::memory_order_relaxed);
                continue;
            }
            node->state.store(kExpanding, std::memory_order_relaxed);
            g.encode_bits(group_.words.data() + (size_t)n * words_);
            g.legal_mask(group_.legal.data() + (size_t)n * actions_);
            group_.leaves[n] = node;
            ++n;
        }
        if (n == 0) continue;
        evaluator_->evaluate_packed_group(group_.word_ptrs.data(), n, words_, group_.policy_ptrs.data(),
                                          group_.values.data());
        for (int i = 0; i < n; ++i) {
            expand(group_.leaves[i], group_.policy_ptrs[i], group_.legal.data() + (size_t)i * actions_,
                   arena);
            group_.leaves[i]->state.store(kExpanded, std::memory_order_relaxed);
            backup(group_.paths[i], group_.values[i]);
            ++done;
            playouts_.fetch_add(1, std::memory_order_relaxed);
        }
    }
    sims_done_.store(done, std::memory_order_relaxed);
}

void FastSearch::worker_loop(int tid) {
    uint64_t seen = 0;
    for (;;) {
        {
            std::unique_lock<std::mutex> lock(mu_);
            cv_.wait(lock, [&] { return stop_ || generation_ != seen; });
            if (stop_) return;
            seen = generation_;
        }
        playouts_from_root(tid);
        {
            std::lock_guard<std::mutex> lock(mu_);
            ++finished_;
        }
        cv_.notify_all();
    }
}

// MCTS::search (src/mcts.cpp:261-325).
void FastSearch::search(const GoPosition& pos, std::vector<float>& visits, bool add_noise) {
    if (pos.size() != board_) throw std::invalid_argument("FastSearch: board size mismatch");
    // The pool is idle between searches: every arena starts over (the
    // previous search's tree is gone with its root).
    for (Arena& a : arenas_) a.reset();
    std::unique_ptr<Node> root(new Node);
    {
        std::vector<uint32_t> words(words_);
        std::vector<float> policy(actions_);
        std::vector<uint8_t> legal(actions_);
        float value = 0.0f;
        pos.encode_bits(words.data());
        evaluator_->evaluate_packed(words.data(), words_, policy.data(), &value);
        pos.legal_mask(legal.data());
        expand(root.get(), policy.data(), legal.data(), arenas_[0]);
        root->state.store(kExpanded, std::memory_order_release);
        root->visits.store(1, std::memory_order_relaxed);
        root->add_value(value);
        if (add_noise) add_dirichlet_noise(root.get());
    }
    pos_ = &pos;
    root_ = root.get();
    sims_done_.store(0, std::memory_order_relaxed);
    if (params_.grouped) {
        grouped_playouts();
        root_ = nullptr;
        pos_ = nullptr;
        visits.assign(actions_, 0.0f);
        for (int i = 0; i < root->n_children; ++i)
            visits[root->children[i].action] =
                (float)root->children[i].visits.load(std::memory_order_relaxed);
        return;
    }
    {
        std::lock_guard<std::mutex> lock(mu_);
        finished_ = 0;
        error_ = nullptr;
        ++generation_;
    }
    cv_.notify_all();
    playouts_from_root(0);
    std::exception_ptr err;
    {
        std::unique_lock<std::mutex> lock(mu_);
        cv_.wait(lock, [&] { return finished_ == (int)pool_.size(); });
        err = error_;
    }
    root_ = nullptr;
    pos_ = nullptr;
    if (err) std::rethrow_exception(err);
    visits.assign(actions_, 0.0f);
    for (int i = 0; i < root->n_children; ++i)
        visits[root->children[i].action] =
            (float)root->children[i].visits.load(std::memory_order_relaxed);
}

// MCTS::get_action (src/mcts.cpp:327-359).
int FastSearch::get_action(const GoPosition& pos, std::vector<float>& policy, float temperature,
                           bool add_noise) {
    std::vector<float> visits;
    search(pos, visits, add_noise);
    if (temperature == 0.0f) {
        const int best = (int)(std::max_element(visits.begin(), visits.end()) - visits.begin());
        policy.assign(actions_, 0.0f);
        policy[best] = 1.0f;
        return best;
    }
    policy.resize(actions_);
    float sum = 0.0f;
    for (int a = 0; a < actions_; ++a) {
        policy[a] = std::pow(visits[a], 1.0f / temperature);
        sum += policy[a];
    }
    if (sum > 0.0f) {
        for (auto& p : policy) p /= sum;
    } else {
        std::vector<uint8_t> legal(actions_);
        pos.legal_mask(legal.data());
        float ls = 0.0f;
        for (int a = 0; a < actions_; ++a) ls += (float)legal[a];
        for (int a = 0; a < actions_; ++a) policy[a] = (float)legal[a] / ls;
    }
    std::discrete_distribution<int> dist(policy.begin(), policy.end());
    return dist(rng_);
}

}  // namespace mgb
