// The ggml plugin's graph_compute dispatch (adapters/ggml-rocknpu/src/
// ggml-rocknpu.cpp:978-1650 and rocknpu_mtile_group :838-976), restated as a
// planner over a plain node list: it decides which C-ABI call serves each
// node -- same-input concatenated groups, the QKV stash of prompt batches,
// the decode triple / FFN pair / V-K pair, the FFN composite, the output
// head split, chunked M=16 batches, the M=16 router's CPU fallback -- and
// reports the calls instead of making them.  State the plugin keeps across
// splits and graph evaluations lives in rocknpu_graph_state.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

#include "../../include/rocknpu_b200.h"

namespace {

constexpr size_t kMaxLayers = 256;  // ROCKNPU_QKV_MAX_LAYERS (:23)

// rocknpu_env_enabled / _default (:261-272).
bool env_on(const char* name) {
    const char* v = std::getenv(name);
    return v != nullptr && v[0] != '\0' && v[0] != '0';
}
bool env_default(const char* name, bool dflt) {
    const char* v = std::getenv(name);
    if (v == nullptr || v[0] == '\0') return dflt;
    return v[0] != '0';
}

bool is_q46(int32_t t) { return t == ROCKNPU_GGML_Q4_K || t == ROCKNPU_GGML_Q6_K; }
bool is_quant(int32_t t) { return is_q46(t) || t == ROCKNPU_GGML_Q5_K; }

long long k_of(const rocknpu_graph_node& n) { return n.desc.weight_ne[0]; }
long long n_of(const rocknpu_graph_node& n) { return n.desc.weight_ne[1]; }
long long m_of(const rocknpu_graph_node& n) { return n.desc.act_ne[1]; }

bool name_has(const rocknpu_graph_node& n, const char* needle) {
    return n.weight_name != nullptr && std::strstr(n.weight_name, needle) != nullptr;
}

// rocknpu_attention_layer (:506-516): the weight's name contains `needle`
// and starts with "blk.<layer>." for a layer below kMaxLayers.
bool attention_layer(const rocknpu_graph_node& n, const char* needle, size_t* layer) {
    if (!name_has(n, needle)) return false;
    size_t parsed = 0;
    if (std::sscanf(n.weight_name, "blk.%zu.", &parsed) != 1 || parsed >= kMaxLayers) return false;
    *layer = parsed;
    return true;
}

// The identity of a weight the layer state remembers (rocknpu_qkv_weight_ref).
struct WeightRef {
    const void* data = nullptr;
    size_t bytes = 0;
    int32_t kind = 0;  // 4 / 6
    int32_t has_w8 = 0;
    bool same(const WeightRef& o) const { return data == o.data && bytes == o.bytes && kind == o.kind; }
};

int32_t quant_kind(int32_t t) { return t == ROCKNPU_GGML_Q4_K ? 4 : t == ROCKNPU_GGML_Q6_K ? 6 : 0; }

WeightRef ref_of(const rocknpu_graph_node& n) {
    WeightRef r;
    r.data = n.weight;
    r.bytes = n.weight_bytes;
    r.kind = quant_kind(n.desc.weight_type);
    r.has_w8 = n.has_w8;
    return r;
}

// rocknpu_qkv_layer_state (:32-53): decode triple (q, v, k refs, stability,
// pending V/K outputs) and the prompt-batch stash (K/V weights seen, pending
// K/V outputs for the activation and row count the Q node ran with).
struct LayerState {
    WeightRef q, v, k;
    size_t stable_observations = 0;
    const void* activation = nullptr;
    bool pending = false;
    // prompt batches
    const void* mk_weight = nullptr;
    long long mk_k = 0, mk_n = 0;
    int32_t mk_type = 0;
    const void* mv_weight = nullptr;
    long long mv_k = 0, mv_n = 0;
    int32_t mv_type = 0;
    long long mk_out = 0, mv_out = 0;  // sizes (m * n) of the stashed outputs
    const void* m_activation = nullptr;
    long long m_rows = 0;
    bool mk_pending = false, mv_pending = false, m_released = false;
};

}  // namespace

struct rocknpu_graph_state {
    bool cpu_fallback = false;
    LayerState qkv[kMaxLayers];
    // FFN composite (rocknpu_backend_context ffn_composite_*, :1300-1318)
    bool ffn_pending = false;
    long long ffn_k = 0, ffn_n = 0;
    const void* ffn_gate = nullptr;
    const void* ffn_up = nullptr;
};

namespace {

// Output of one planning pass.
struct Plan {
    rocknpu_graph_action* out;
    size_t cap;
    size_t used = 0;
    bool overflow = false;
    rocknpu_graph_action& add(int32_t call, int32_t node) {
        static rocknpu_graph_action sink;
        if (used >= cap) {
            overflow = true;
            return sink;
        }
        rocknpu_graph_action& a = out[used++];
        std::memset(&a, 0, sizeof(a));
        a.call = call;
        a.node = node;
        a.layer = -1;
        for (int i = 0; i < 4; ++i) a.members[i] = -1;
        return a;
    }
};

void set_member(rocknpu_graph_action& a, int slot, int32_t node, const void* weight) {
    a.members[slot] = node;
    a.weights[slot] = weight;
    if (slot + 1 > a.count) a.count = slot + 1;
}

// rocknpu_mtile_group_m1_candidate (:846-859): a prompt-sized K-quant
// projection that may join a same-input group.
bool group_candidate(const rocknpu_graph_node& n) {
    if (!env_default("ROCKNPU_MTILE_GROUP", true) || n.op != ROCKNPU_OP_MUL_MAT || !n.desc.is_mul_mat) return false;
    const rocknpu_mul_mat_desc& d = n.desc;
    if (!is_q46(d.weight_type)) return false;
    const long long m = d.act_ne[1], k = d.weight_ne[0];
    return m >= 32 && d.act_type == ROCKNPU_GGML_F32 && d.dst_type == ROCKNPU_GGML_F32 && d.act_contiguous &&
           d.dst_contiguous && d.act_ne[2] == 1 && d.act_ne[3] == 1 && k % 512 == 0 && k <= 4096 &&
           d.weight_ne[1] % 32 == 0;
}

bool supported(const rocknpu_graph_node& n) { return rocknpu_mul_mat_supported(&n.desc) != 0; }

// rocknpu_mtile_group (:861-976): the node at `first` together with later
// nodes of the split reading the same activations, as one concatenated-N
// call -- or the layer's stashed K/V outputs, or Q run together with the
// layer's K and V.  Returns how many projections it served (0 = none).
int mtile_group(rocknpu_graph_state* st, const rocknpu_graph_node* nodes, size_t count, size_t first,
                std::vector<char>& done, Plan& plan) {
    const rocknpu_graph_node& lead = nodes[first];
    size_t members[4] = {first, 0, 0, 0};
    int n_members = 1;
    for (size_t j = first + 1; j < count && n_members < 4; ++j) {
        const rocknpu_graph_node& c = nodes[j];
        if (!c.compute) continue;
        if (c.op == ROCKNPU_OP_MUL_MAT && c.activation == lead.activation && k_of(c) == k_of(lead) &&
            group_candidate(c) && supported(c))
            members[n_members++] = j;
    }
    const bool qkv_enabled = env_default("ROCKNPU_MTILE_QKV", true);
    const long long m = m_of(lead), k = k_of(lead);
    size_t layer = 0;
    if (qkv_enabled) {
        // remember each layer's K/V weights; serve K/V from the stash the Q
        // node left when every member is stashed
        int stashed = 0;
        for (int g = 0; g < n_members; ++g) {
            const rocknpu_graph_node& w = nodes[members[g]];
            if (attention_layer(w, ".attn_k.weight", &layer)) {
                LayerState& s = st->qkv[layer];
                s.mk_weight = w.weight;
                s.mk_k = k_of(w);
                s.mk_n = n_of(w);
                s.mk_type = w.desc.weight_type;
                stashed += s.mk_pending && s.m_activation == lead.activation_data && s.m_rows == m &&
                           s.mk_out == m * n_of(w);
            } else if (attention_layer(w, ".attn_v.weight", &layer)) {
                LayerState& s = st->qkv[layer];
                s.mv_weight = w.weight;
                s.mv_k = k_of(w);
                s.mv_n = n_of(w);
                s.mv_type = w.desc.weight_type;
                stashed += s.mv_pending && s.m_activation == lead.activation_data && s.m_rows == m &&
                           s.mv_out == m * n_of(w);
            }
        }
        if (stashed == n_members) {
            for (int g = 0; g < n_members; ++g) {
                const rocknpu_graph_node& w = nodes[members[g]];
                const bool is_k = attention_layer(w, ".attn_k.weight", &layer);
                if (!is_k) attention_layer(w, ".attn_v.weight", &layer);
                LayerState& s = st->qkv[layer];
                (is_k ? s.mk_pending : s.mv_pending) = false;
                rocknpu_graph_action& a = plan.add(ROCKNPU_CALL_STASH, static_cast<int32_t>(members[g]));
                set_member(a, 0, static_cast<int32_t>(members[g]), w.weight);
                a.layer = static_cast<int32_t>(layer);
                a.m = m;
                a.k = k;
                a.n = n_of(w);
                if (g > 0) done[members[g]] = 1;
            }
            return n_members;
        }
    }
    // Q of a layer whose K/V weights are known: Q, K and V together
    const void* weights[4] = {};
    long long ns[4] = {};
    int32_t kinds[4] = {};
    int32_t idx[4] = {-1, -1, -1, -1};
    for (int g = 0; g < n_members; ++g) {
        weights[g] = nodes[members[g]].weight;
        ns[g] = n_of(nodes[members[g]]);
        kinds[g] = nodes[members[g]].desc.weight_type;
        idx[g] = static_cast<int32_t>(members[g]);
    }
    LayerState* q_state = nullptr;
    if (qkv_enabled && n_members == 1 && attention_layer(lead, ".attn_q.weight", &layer)) {
        LayerState& s = st->qkv[layer];
        s.mk_pending = s.mv_pending = false;
        if (s.mk_weight != nullptr && s.mv_weight != nullptr && s.mk_k == k && s.mv_k == k) {
            s.mk_out = m * s.mk_n;
            s.mv_out = m * s.mv_n;
            weights[1] = s.mk_weight;
            ns[1] = s.mk_n;
            kinds[1] = s.mk_type;
            weights[2] = s.mv_weight;
            ns[2] = s.mv_n;
            kinds[2] = s.mv_type;
            idx[1] = idx[2] = -1;
            q_state = &s;
            n_members = 3;
        }
    }
    long long total_n = 0;
    for (int g = 0; g < n_members; ++g) total_n += ns[g];
    if (n_members == 1) return 0;  // a single wide projection keeps its own path
    if (total_n > 3 * 8192) return 0;
    for (int g = 0; g < n_members; ++g)
        if (!is_q46(kinds[g])) return 0;
    rocknpu_graph_action& a = plan.add(ROCKNPU_CALL_CONCAT, static_cast<int32_t>(first));
    for (int g = 0; g < n_members; ++g) set_member(a, g, idx[g], weights[g]);
    a.m = m;
    a.k = k;
    a.n = total_n;
    if (q_state != nullptr) {
        a.layer = static_cast<int32_t>(layer);
        q_state->m_activation = lead.activation_data;
        q_state->m_rows = m;
        q_state->mk_pending = q_state->mv_pending = true;
        if (!q_state->m_released) {
            // the single/pair prompt caches of these weights are now unused
            const int32_t layer_of_call = a.layer;
            rocknpu_graph_action& r = plan.add(ROCKNPU_CALL_RELEASE, static_cast<int32_t>(first));
            for (int g = 0; g < 3; ++g) set_member(r, g, idx[g], weights[g]);
            r.layer = layer_of_call;
            q_state->m_released = true;
        }
    }
    for (int g = 1; g < n_members; ++g)
        if (q_state == nullptr) done[members[g]] = 1;
    return n_members;
}

// rocknpu_small_native_mtile_supported (:290-303) and friends, for the M=16
// router and the chunked-batch switches.
bool w8_shape(long long k, long long n) {
    if (!env_on("ROCKNPU_W8_MTILE")) return false;
    const char* scope = std::getenv("ROCKNPU_W8_MTILE_SCOPE");
    if (scope == nullptr || scope[0] == '\0' || !std::strcmp(scope, "all")) return true;
    if (!std::strcmp(scope, "kv")) return k == 2048 && n == 256;
    if (!std::strcmp(scope, "qo")) return k == 2048 && n == 2048;
    if (!std::strcmp(scope, "ffn")) return (k == 2048 && n == 5632) || (k == 5632 && n == 2048);
    if (!std::strcmp(scope, "attn")) return k == 2048 && (n == 256 || n == 2048);
    if (!std::strcmp(scope, "safe")) return k == 2048 && (n == 256 || n == 5632);
    return false;
}
bool small_native(long long m, long long k, long long n) {
    if (!(m == 4 || m == 8 || m == 12) || !env_on("ROCKNPU_NATIVE_MTILE") || !env_on("ROCKNPU_MTILE_PERSIST") ||
        !w8_shape(k, n))
        return false;
    if (k == 5632 && n == 2048) return env_on("ROCKNPU_NATIVE_MTILE_DOWN") && env_on("ROCKNPU_MTILE_MC");
    return k > 0 && k <= 4096 && k % 512 == 0 && n > 0 && n <= 8192 && n % 32 == 0;
}

// The M=16 router (:980-1068): with a CPU fallback backend, a split whose
// MUL_MATs are not all M=16-routable (or, under ROCKNPU_RUNTIME_M16_W8_ONLY,
// not all W8-shaped; or any forced-CPU shape) goes to the CPU, after
// pre-warming the prompt caches of the TinyLlama shapes when asked to.
bool route_to_cpu(const rocknpu_graph_node* nodes, size_t count, Plan& plan) {
    bool has_mul_mat = false, all_m16 = true, all_w8_m16 = true, force_cpu = false;
    const bool split_m32 = env_on("ROCKNPU_M32_AS_2X16"), chunk_m16 = env_on("ROCKNPU_M16_CHUNK_BATCH");
    const bool native_mtile = env_on("ROCKNPU_NATIVE_MTILE"), prewarm = env_on("ROCKNPU_RUNTIME_M16_PREWARM");
    const bool cpu_kv = env_on("ROCKNPU_RUNTIME_CPU_KV"), cpu_qo = env_on("ROCKNPU_RUNTIME_CPU_QO"),
               cpu_ffn = env_on("ROCKNPU_RUNTIME_CPU_FFN");
    std::vector<size_t> prewarm_nodes;
    for (size_t i = 0; i < count; ++i) {
        const rocknpu_graph_node& nd = nodes[i];
        if (!nd.compute || nd.op != ROCKNPU_OP_MUL_MAT) continue;
        has_mul_mat = true;
        const int32_t wt = nd.desc.weight_type;
        const bool quantized = is_quant(wt);
        const long long m = m_of(nd), k = k_of(nd), n = n_of(nd);
        if (prewarm && quantized && ((k == 2048 && (n == 256 || n == 2048 || n == 5632)) || (k == 5632 && n == 2048)))
            prewarm_nodes.push_back(i);
        const bool native_small = quantized && small_native(m, k, n);
        const bool q5_chunked = native_mtile && wt == ROCKNPU_GGML_Q5_K && m > 1;
        const bool native_batch =
            native_small || q5_chunked || (native_mtile && quantized && m >= 32 && m <= 128 && m % 16 == 0);
        const bool routed = m == 16 || native_batch || (split_m32 && m == 32) ||
                            (chunk_m16 && m >= 32 && m <= 128 && m % 16 == 0);
        if (!routed) all_m16 = false;
        const bool w8 = quantized && (m == 16 || native_batch) && k > 0 && k <= 4096 && k % 512 == 0 && n > 0 &&
                        n <= 8192 && n % 32 == 0;
        all_w8_m16 = all_w8_m16 && w8;
        if (quantized && routed && k == 2048) {
            force_cpu = force_cpu || (cpu_kv && n == 256);
            force_cpu = force_cpu || (cpu_qo && n == 2048);
            force_cpu = force_cpu || (cpu_ffn && n == 5632);
        }
    }
    const bool w8_only = env_on("ROCKNPU_RUNTIME_M16_W8_ONLY");
    if (!(has_mul_mat && (!all_m16 || (w8_only && !all_w8_m16) || force_cpu))) return false;
    for (size_t i : prewarm_nodes) {
        if (!is_q46(nodes[i].desc.weight_type)) continue;
        rocknpu_graph_action& a = plan.add(ROCKNPU_CALL_PREWARM, static_cast<int32_t>(i));
        set_member(a, 0, static_cast<int32_t>(i), nodes[i].weight);
        a.m = 16;
        a.k = k_of(nodes[i]);
        a.n = n_of(nodes[i]);
    }
    plan.add(ROCKNPU_CALL_CPU_FALLBACK, -1);
    return true;
}

void single(const rocknpu_graph_node& nd, size_t i, int32_t call, int32_t w8, Plan& plan) {
    rocknpu_graph_action& a = plan.add(call, static_cast<int32_t>(i));
    set_member(a, 0, static_cast<int32_t>(i), nd.weight);
    a.w8 = w8;
    a.m = m_of(nd);
    a.k = k_of(nd);
    a.n = n_of(nd);
}

// One split (:1069-1650).
void plan_split(rocknpu_graph_state* st, const rocknpu_graph_node* nodes, size_t count, Plan& plan) {
    if (st->cpu_fallback && route_to_cpu(nodes, count, plan)) return;
    std::vector<char> done(count, 0);  // served by an earlier same-input group
    for (size_t i = 0; i < count; ++i) {
        const rocknpu_graph_node& nd = nodes[i];
        if (!nd.compute || done[i]) continue;
        if (nd.op == ROCKNPU_OP_VIEW) continue;
        if (nd.op != ROCKNPU_OP_MUL_MAT || !supported(nd)) {
            plan.add(ROCKNPU_CALL_FAILED, static_cast<int32_t>(i));
            return;
        }
        if (group_candidate(nd) && mtile_group(st, nodes, count, i, done, plan) > 0) continue;
        const long long m = m_of(nd), k = k_of(nd), n = n_of(nd);
        const int32_t wt = nd.desc.weight_type;
        // the output head at M=1 through the W8 sidecar, 8192 columns a chunk
        if (env_on("ROCKNPU_NPU_OUTPUT_HEAD") && m == 1 && n > 8192 && name_has(nd, "output.weight") && is_q46(wt)) {
            if (!nd.has_w8) {
                plan.add(ROCKNPU_CALL_FAILED, static_cast<int32_t>(i));
                return;
            }
            single(nd, i, ROCKNPU_CALL_OUTPUT_HEAD_NSPLIT, 1, plan);
            continue;
        }
        // the FFN composite: down after a deferred gate/up pair
        if (env_on("ROCKNPU_FFN_COMPOSITE") && st->ffn_pending && m == 1 && k == st->ffn_n && n == 2048 &&
            name_has(nd, ".ffn_down.weight") && is_q46(wt) && nd.has_w8) {
            rocknpu_graph_action& a = plan.add(ROCKNPU_CALL_SWIGLU_DOWN, static_cast<int32_t>(i));
            set_member(a, 0, -1, st->ffn_gate);
            set_member(a, 1, -1, st->ffn_up);
            set_member(a, 2, static_cast<int32_t>(i), nd.weight);
            a.w8 = 1;
            a.m = 1;
            a.k = st->ffn_k;
            a.n = n;
            st->ffn_pending = false;
            continue;
        }
        // decode Q of a layer whose V and K have been seen twice unchanged:
        // Q, V and K as one call (V and K kept for their own nodes)
        size_t layer = 0;
        if (env_default("ROCKNPU_QKV_TRIPLE", true) && attention_layer(nd, ".attn_q.weight", &layer) && m == 1 &&
            k == 2048 && n == 2048 && is_q46(wt)) {
            LayerState& s = st->qkv[layer];
            const WeightRef cur = ref_of(nd);
            if (!s.q.same(cur)) {
                s.q = cur;
                s.stable_observations = 0;
                s.pending = false;
            } else if (s.stable_observations >= 2 && s.v.data != nullptr && s.k.data != nullptr) {
                s.pending = false;
                const bool w8 = nd.has_w8 && s.v.has_w8 && s.k.has_w8;
                rocknpu_graph_action& a = plan.add(ROCKNPU_CALL_TRIPLE_M1, static_cast<int32_t>(i));
                set_member(a, 0, static_cast<int32_t>(i), nd.weight);
                set_member(a, 1, -1, s.v.data);
                set_member(a, 2, -1, s.k.data);
                a.w8 = w8;
                a.layer = static_cast<int32_t>(layer);
                a.m = 1;
                a.k = 2048;
                a.n = 2048 + 256 + 256;
                s.activation = nd.activation_data;
                s.pending = true;
                continue;
            }
        }
        // gate at i, up at i + 1 on the same activations
        if (env_default("ROCKNPU_FFN_PAIR", true) && i + 1 < count) {
            const rocknpu_graph_node& up = nodes[i + 1];
            if (up.op == ROCKNPU_OP_MUL_MAT && supported(up)) {
                const bool native_pair = (m == 4 || m == 8 || m == 12 || m == 16) && env_on("ROCKNPU_NATIVE_MTILE") &&
                                         env_on("ROCKNPU_W8_MTILE") && env_on("ROCKNPU_MTILE_PERSIST") &&
                                         env_on("ROCKNPU_MTILE_MC");
                const bool ffn_pair = name_has(nd, ".ffn_gate.weight") && name_has(up, ".ffn_up.weight") &&
                                      nd.activation == up.activation && (m == 1 || native_pair) && k == k_of(up) &&
                                      n == 5632 && n_of(up) == 5632 && is_q46(wt) && is_q46(up.desc.weight_type);
                if (ffn_pair) {
                    const bool w8 = m == 1 && nd.has_w8 && up.has_w8;
                    if (m == 1 && w8 && env_on("ROCKNPU_FFN_COMPOSITE")) {
                        st->ffn_pending = true;
                        st->ffn_k = k;
                        st->ffn_n = 5632;
                        st->ffn_gate = nd.weight;
                        st->ffn_up = up.weight;
                        rocknpu_graph_action& a = plan.add(ROCKNPU_CALL_FFN_DEFER, static_cast<int32_t>(i));
                        set_member(a, 0, static_cast<int32_t>(i), nd.weight);
                        set_member(a, 1, static_cast<int32_t>(i + 1), up.weight);
                        a.w8 = 1;
                        a.m = 1;
                        a.k = k;
                        a.n = 2 * 5632;
                        ++i;
                        continue;
                    }
                    rocknpu_graph_action& a =
                        plan.add(m == 1 ? ROCKNPU_CALL_PAIR_M1 : ROCKNPU_CALL_PAIR_MTILE, static_cast<int32_t>(i));
                    set_member(a, 0, static_cast<int32_t>(i), nd.weight);
                    set_member(a, 1, static_cast<int32_t>(i + 1), up.weight);
                    a.w8 = w8;
                    a.m = m;
                    a.k = k;
                    a.n = 2 * 5632;
                    ++i;
                    continue;
                }
            }
        }
        // decode V at i, K at i + 2: from the layer's triple stash, or a pair
        if (env_default("ROCKNPU_VK_PAIR", true) && i + 2 < count) {
            const rocknpu_graph_node& kn = nodes[i + 2];
            if (kn.op == ROCKNPU_OP_MUL_MAT && supported(kn)) {
                const bool vk = name_has(nd, ".attn_v.weight") && name_has(kn, ".attn_k.weight") &&
                                nd.activation == kn.activation && m == 1 && k == k_of(kn) && n == 256 &&
                                n_of(kn) == 256 && is_q46(wt) && is_q46(kn.desc.weight_type);
                if (vk) {
                    bool served = false;
                    if (attention_layer(nd, ".attn_v.weight", &layer)) {
                        LayerState& s = st->qkv[layer];
                        const WeightRef cv = ref_of(nd), ck = ref_of(kn);
                        const bool same = s.v.same(cv) && s.k.same(ck);
                        s.v = cv;
                        s.k = ck;
                        s.stable_observations = same ? s.stable_observations + 1 : 1;
                        if (env_default("ROCKNPU_QKV_TRIPLE", true) && s.pending) {
                            if (s.activation == nd.activation_data) {
                                rocknpu_graph_action& a = plan.add(ROCKNPU_CALL_STASH, static_cast<int32_t>(i));
                                set_member(a, 0, static_cast<int32_t>(i), nd.weight);
                                set_member(a, 1, static_cast<int32_t>(i + 2), kn.weight);
                                a.layer = static_cast<int32_t>(layer);
                                a.m = 1;
                                a.k = k;
                                a.n = 512;
                                served = true;
                            }
                            s.pending = false;
                        }
                    }
                    if (!served) {
                        rocknpu_graph_action& a = plan.add(ROCKNPU_CALL_PAIR_M1, static_cast<int32_t>(i));
                        set_member(a, 0, static_cast<int32_t>(i), nd.weight);
                        set_member(a, 1, static_cast<int32_t>(i + 2), kn.weight);
                        a.w8 = nd.has_w8 && kn.has_w8;
                        a.m = 1;
                        a.k = k;
                        a.n = 512;
                    }
                    i += 2;
                    continue;
                }
            }
        }
        // one node: chunked into 16-row calls, or a single call
        const bool quantized = is_quant(wt);
        const bool native_mtile = quantized && (small_native(m, k, n) ||
                                                (wt == ROCKNPU_GGML_Q5_K && m > 1 && env_on("ROCKNPU_NATIVE_MTILE")) ||
                                                (m >= 32 && m <= 128 && m % 16 == 0 && env_on("ROCKNPU_NATIVE_MTILE")));
        const bool split_m32 = !native_mtile && m == 32 && env_on("ROCKNPU_M32_AS_2X16");
        const bool chunked = !native_mtile && m >= 32 && m <= 128 && m % 16 == 0 && env_on("ROCKNPU_M16_CHUNK_BATCH");
        if (split_m32 || chunked) {
            single(nd, i, ROCKNPU_CALL_CHUNKED_M16, 0, plan);
            continue;
        }
        single(nd, i, ROCKNPU_CALL_SINGLE, m == 1 && nd.has_w8 ? 1 : 0, plan);
    }
}

}  // namespace

extern "C" {

rocknpu_graph_state* rocknpu_graph_state_create(int32_t cpu_fallback) {
    auto* s = new (std::nothrow) rocknpu_graph_state();
    if (s) s->cpu_fallback = cpu_fallback != 0;
    return s;
}

void rocknpu_graph_state_destroy(rocknpu_graph_state* state) { delete state; }

int rocknpu_graph_plan(rocknpu_graph_state* state, const rocknpu_graph_node* nodes, size_t count,
                       rocknpu_graph_action* actions, size_t capacity) {
    if (!state || (!nodes && count) || (!actions && capacity)) return -1;
    Plan plan{actions, capacity};
    plan_split(state, nodes, count, plan);
    return plan.overflow ? -1 : static_cast<int>(plan.used);
}

}  // extern "C"
