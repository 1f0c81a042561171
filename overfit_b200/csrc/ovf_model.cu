// ovf_model.cu — device-resident model and decode session behind the C ABI
// (ovf_model_create / ovf_session_*), the GPU counterpart of
// CachedLlamaInferenceEngine + CachedLlamaSession (Runtime/
// CachedLlamaInferenceEngine.cs:33, Runtime/CachedLlamaSession.cs:26).
//
// One decode step is 2 + 4*n_layers kernels, all launched with programmatic
// dependent launch and captured once into a CUDA graph per session:
//   embed(token)                                   EmbedAndAdvance
//   per layer:
//     GEMV  rmsnorm+Q8_K | Wq,Wk,Wv (+bias)        RmsNormalize, ProjectKv/Q
//     ATTN  RoPE(q,k), KV append, flash-decode     RopeKernel, WriteKey/Value, ComputeSingleHead
//     GEMV  Q8_0 Wo per head, + residual           AttendAndProjectO, head-ordered sum, AddResidual
//     GEMV  rmsnorm+Q8_K | gate,up -> silu*up      DecodeSwiGluDispatched (fused gate/up)
//     GEMV  Q8_K | down, + residual                down projection, AddResidual
//   GEMV  rmsnorm | lm head -> logits + argmax     final norm, ProjectLogits, TokenSampler.ArgMax
// The argmax is fed back on the device, so greedy generation replays the
// graph with no host round trip.
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "ovf_internal.cuh"

using namespace ovf;

namespace {

struct DevWeight {
    int type = -1;         // OVF_TYPE_* as resident on the device
    uint8_t *data = nullptr;  // K-quant bytes / Q8_0 int8 quants / f32
    float *scales = nullptr;  // Q8_0 fp32 scales
    int64_t rows = 0, cols = 0;
    bool owns = true;
};

struct DevLayer {
    float *attn_norm = nullptr, *ffn_norm = nullptr;
    DevWeight wq, wk, wv, wo, gate, up, down;
    float *bq = nullptr, *bk = nullptr, *bv = nullptr, *bo = nullptr;
    // MoE (n_experts > 0): F32 router [d_model][n_experts] (input-major, as
    // GgufLlamaLoader.cs:770-786 transposes ffn_gate_inp); gate/up/down hold
    // the experts' matrices back to back, `*_stride` bytes apart
    float *router = nullptr;
    int64_t gu_wstride = 0, gu_sstride = 0, d_wstride = 0, d_sstride = 0;
};

// MoE scratch of a batch of rows (allocated on first use): the routing
// [rows][k], per-expert row lists, the gathered inputs, one expert's outputs
// and every row's k expert outputs [rows][k][d_model].
struct MoeRows {
    int cap = 0;
    int32_t *sel = nullptr, *idx = nullptr;  // idx: rows [E][cap] then slots [E][cap]
    float *w = nullptr, *gx = nullptr, *eo = nullptr, *slot = nullptr;
    int32_t *host = nullptr;  // pinned: sel [cap][k] | rows/slots [2][E][cap]
};

// Bytes of one expert's quants and Q8_0 scales in a stacked expert weight.
void expert_strides(const DevWeight &w, int64_t rows_e, int64_t *wstride, int64_t *sstride) {
    if (w.type == OVF_TYPE_Q8_0) {
        *wstride = rows_e * w.cols;
        *sstride = rows_e * (w.cols / 32) * 4;
    } else {
        *wstride = rows_e * (w.cols / 256) * (w.type == OVF_TYPE_Q4_K ? 144 : 210);
        *sstride = 0;
    }
}

// One expert of a stacked expert weight as a weight of its own.
DevWeight expert_view(const DevWeight &w, int64_t rows_e, int e) {
    int64_t ws = 0, ss = 0;
    expert_strides(w, rows_e, &ws, &ss);
    DevWeight v = w;
    v.data = w.data + (size_t)e * ws;
    v.scales = w.scales ? reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(w.scales) + (size_t)e * ss) : nullptr;
    v.rows = rows_e;
    v.owns = false;
    return v;
}

}  // namespace

struct ovf_model {
    int device = 0;
    ovf_model_config cfg{};
    std::vector<DevLayer> layers;
    DevWeight embed, lm_head;
    float *final_norm = nullptr;
    std::vector<void *> allocs;
    int64_t weight_bytes = 0;
    // multi-session decode scratch (allocated on first use)
    int b_rows = 0;
    float *bx = nullptr, *ba = nullptr, *bn = nullptr, *bq = nullptr, *bk = nullptr, *bv = nullptr, *batt = nullptr,
          *bg = nullptr, *bu = nullptr, *bh = nullptr, *bas = nullptr, *blogits = nullptr;
    int8_t *baq = nullptr;
    int16_t *bab = nullptr;
    int32_t *btok = nullptr, *bargmax = nullptr;
    int32_t *btok_host = nullptr;  // pinned
    std::atomic<bool> batch_busy{false};  // one ovf_session_decode_batch at a time per model
    MoeRows bmoe;                          // MoE scratch of the batch rows
    // tensor parallelism (world > 1): this rank's share of heads, FFN rows
    // and vocabulary; the exchange arena (IPC-exported) and the peers'
    int tp_rank = 0, tp_world = 1;
    int h_loc = 0, kvh_loc = 0, ff_loc = 0, v_loc = 0, nb_down = 0;  // nb_down: down blocks of all ranks
    char *arena = nullptr;
    size_t arena_bytes = 0, off_heads = 0, off_terms = 0, off_logits = 0, off_keys = 0, off_flags = 0, off_epoch = 0,
           off_moe = 0;
    char *peer[8] = {};
    bool tp_ready = false;
};

struct ovf_session {
    ovf_model *m = nullptr;
    int max_ctx = 0;
    int pos = 0;           // host mirror of DevStep::next_pos
    bool needs_reset = false;  // a batch call failed after touching this session's state
    bool prefill_single = false;  // DisableBatchedPrefillForParity
    int n_logits = 0;      // host mirror of DevStep::n_generated
    cudaStream_t stream = nullptr;
    int kv_dtype = OVF_KV_F32;
    void *kc = nullptr, *vc = nullptr;  // [layers][KVH][max_ctx][hd], fp32, int8 or fp16
    float *ks = nullptr, *vs = nullptr;  // Q8 cache: scales [layers][KVH][max_ctx]
    float *hidden = nullptr, *after = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *attn = nullptr, *h = nullptr,
          *gtmp = nullptr, *utmp = nullptr, *logits = nullptr, *rope_cos = nullptr, *rope_sin = nullptr,
          *partial = nullptr;
    int *counters = nullptr, *tokens_log = nullptr;
    int *err_slot = nullptr;  // device word the error word is moved into after a call
    int32_t *msel = nullptr;  // MoE decode: selected experts [k], their weights [k],
    float *mw = nullptr, *mh = nullptr, *meo = nullptr;  // SwiGLU rows [k][d_ff], expert outputs [k][d_model]
    float *norm_s = nullptr;  // [0]: RMSNorm scale of hidden, [1]: of after
    TraceSlot *trace = nullptr;  // OVF_TRACE=1: per-launch timeline of the last step
    int trace_cap = 0, trace_n = 0;
    std::vector<std::string> trace_labels;
    DevStep *step = nullptr;
    int32_t *pinned_tok = nullptr;  // host staging
    int pinned_cap = 0;
    cudaGraphExec_t graph_logits = nullptr, graph_nologits = nullptr;
    // batched prefill scratch (allocated on first use): rows of one chunk
    int pf_rows = 0;
    float *px = nullptr, *pa = nullptr, *pn = nullptr, *pq = nullptr, *pk = nullptr, *pv = nullptr, *patt = nullptr,
          *pg = nullptr, *pu = nullptr, *ph = nullptr, *pas = nullptr, *pscale = nullptr;
    int8_t *paq = nullptr;
    int16_t *pab = nullptr;
    void *ptc = nullptr;  // packed operands of the tensor-core Q4_K projection
    int32_t *ptok = nullptr;
    MoeRows pmoe;  // MoE scratch of the prefill rows
    float *pattn = nullptr;  // prefill attention: p_t of every (row, head) of a chunk [rows][heads][max_ctx]
    // speculative verify: per-row logits and argmax of one verify batch
    float *vlogits = nullptr;
    int32_t *vargmax = nullptr;
    std::vector<void *> allocs;
};

namespace {

ovf_status dalloc(std::vector<void *> &list, void **p, size_t bytes) {
    if (bytes == 0) bytes = 16;
    cudaError_t e = cudaMalloc(p, bytes);
    if (e != cudaSuccess) return cuda_status(e, "cudaMalloc");
    list.push_back(*p);
    return OVF_OK;
}

ovf_status moe_rows_alloc(const ovf_model_config &c, int cap, std::vector<void *> &allocs, MoeRows *mr) {
    if (mr->cap >= cap) return OVF_OK;
    const size_t K = c.n_experts_used, E = c.n_experts, D = c.d_model;
    ovf_status st = OVF_OK;
    auto A = [&](void **p, size_t bytes) {
        if (!st) st = dalloc(allocs, p, bytes);
    };
    A((void **)&mr->sel, cap * K * 4);
    A((void **)&mr->idx, 2 * E * cap * 4);
    A((void **)&mr->w, cap * K * 4);
    A((void **)&mr->gx, cap * D * 4);
    A((void **)&mr->eo, cap * D * 4);
    A((void **)&mr->slot, cap * K * D * 4);
    if (!st) st = cuda_status(cudaMallocHost(&mr->host, (cap * K + 2 * E * cap) * 4), "cudaMallocHost");
    if (!st) mr->cap = cap;
    return st;
}

int64_t tensor_bytes(int type, int64_t rows, int64_t cols) {
    switch (type) {
        case OVF_TYPE_F32: return rows * cols * 4;
        case OVF_TYPE_Q8_0: return rows * cols / 32 * 34;
        case OVF_TYPE_Q4_K: return rows * cols / 256 * 144;
        case OVF_TYPE_Q6_K: return rows * cols / 256 * 210;
        default: return -1;
    }
}

int64_t host_row_bytes(int type, int64_t cols) {
    switch (type) {
        case OVF_TYPE_F32: return cols * 4;
        case OVF_TYPE_Q8_0: return cols / 32 * 34;
        case OVF_TYPE_Q4_K: return cols / 256 * 144;
        case OVF_TYPE_Q6_K: return cols / 256 * 210;
        default: return -1;
    }
}

// Rows [r0, r0 + n) of a host tensor (a view, no copy).
ovf_tensor host_rows(const ovf_tensor &t, int64_t r0, int64_t n) {
    ovf_tensor v = t;
    if (t.data) v.data = static_cast<const char *>(t.data) + r0 * host_row_bytes(t.type, t.cols);
    v.rows = n;
    return v;
}

// Columns [k0, k0 + kn) of every row of a host tensor, gathered into `buf`
// (k0, kn multiples of the block length).
ovf_tensor host_cols(const ovf_tensor &t, int64_t k0, int64_t kn, std::vector<uint8_t> &buf) {
    const int64_t rb = host_row_bytes(t.type, t.cols), ob = host_row_bytes(t.type, k0), nb = host_row_bytes(t.type, kn);
    buf.resize((size_t)(t.rows * nb));
    for (int64_t r = 0; r < t.rows; ++r)
        memcpy(buf.data() + r * nb, static_cast<const char *>(t.data) + r * rb + ob, (size_t)nb);
    ovf_tensor v{t.type, buf.data(), t.rows, kn};
    return v;
}

// A slice [i0, i0 + n) of an F32 vector tensor.
ovf_tensor host_vec_slice(const ovf_tensor &t, int64_t i0, int64_t n) {
    ovf_tensor v = t;
    if (t.data) v.data = static_cast<const float *>(t.data) + i0;
    v.rows = 1;
    v.cols = n;
    return v;
}

// Uploads an f32 vector (norm / bias).
ovf_status upload_vec(ovf_model *m, const ovf_tensor &t, int64_t n, float **out, const char *what) {
    *out = nullptr;
    if (!t.data) return OVF_OK;
    OVF_CHECK_ARG(t.type == OVF_TYPE_F32, "%s must be F32", what);
    OVF_CHECK_ARG(t.rows * t.cols == n, "%s has %lld elements, expected %lld", what, (long long)(t.rows * t.cols),
                  (long long)n);
    ovf_status st = dalloc(m->allocs, (void **)out, n * 4);
    if (st) return st;
    OVF_CUDA_TRY(cudaMemcpy(*out, t.data, n * 4, cudaMemcpyHostToDevice));
    return OVF_OK;
}

// Uploads a matrix following the reference's residency rules
// (GgufLlamaLoader.cs:941-1203): K-quants stay verbatim; Q8_0 is
// de-interleaved to int8 + fp32 scales; everything else, and any matrix
// `force_q8` asks for (attn_output), becomes Q8_0 with fp32 scales.
ovf_status upload_matrix(ovf_model *m, const ovf_tensor &t, int64_t rows, int64_t cols, bool force_q8, DevWeight *w,
                         const char *what) {
    OVF_CHECK_ARG(t.data, "%s is missing", what);
    OVF_CHECK_ARG(t.rows == rows && t.cols == cols, "%s is %lldx%lld, expected %lldx%lld", what, (long long)t.rows,
                  (long long)t.cols, (long long)rows, (long long)cols);
    const int64_t nbytes = tensor_bytes(t.type, rows, cols);
    OVF_CHECK_ARG(nbytes > 0, "%s has unsupported type %d", what, t.type);
    const bool kq = t.type == OVF_TYPE_Q4_K || t.type == OVF_TYPE_Q6_K;
    OVF_CHECK_ARG(!kq || cols % 256 == 0, "%s: K-quant rows must be multiples of 256", what);
    OVF_CHECK_ARG(cols % 32 == 0, "%s: row length must be a multiple of 32", what);
    void *staging = nullptr;
    ovf_status st = OVF_OK;
    w->rows = rows;
    w->cols = cols;
    if (kq && !force_q8) {
        w->type = t.type;
        st = dalloc(m->allocs, (void **)&w->data, nbytes);
        if (st) return st;
        OVF_CUDA_TRY(cudaMemcpy(w->data, t.data, nbytes, cudaMemcpyHostToDevice));
        m->weight_bytes += nbytes;
        return OVF_OK;
    }
    w->type = OVF_TYPE_Q8_0;
    st = dalloc(m->allocs, (void **)&w->data, rows * cols);
    if (!st) st = dalloc(m->allocs, (void **)&w->scales, rows * cols / 32 * 4);
    if (st) return st;
    m->weight_bytes += rows * cols + rows * cols / 8;
    OVF_CUDA_TRY(cudaMalloc(&staging, nbytes));
    cudaError_t e = cudaMemcpy(staging, t.data, nbytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        if (t.type == OVF_TYPE_Q8_0) st = launch_q8_0_deinterleave(staging, rows * cols, (int8_t *)w->data, w->scales, 0);
        else st = launch_requant_q8_0(t.type, staging, rows, cols, (int8_t *)w->data, w->scales, 0);
        if (!st) e = cudaDeviceSynchronize();
    }
    cudaFree(staging);
    if (e != cudaSuccess) return cuda_status(e, what);
    return st;
}

// Tensor parallelism: the columns [c0, c0 + cn) (this rank's heads) of
// attn_output after the loader's Q8_0 re-quantization of the whole matrix
// (GgufLlamaLoader.cs:977-995: per-head Q8_0 blocks never cross a head).
ovf_status upload_wo_local(ovf_model *m, const ovf_tensor &t, int64_t rows, int64_t cols, int64_t c0, int64_t cn,
                           DevWeight *w) {
    DevWeight full;
    std::vector<void *> keep;
    std::swap(keep, m->allocs);
    const int64_t before = m->weight_bytes;
    ovf_status st = upload_matrix(m, t, rows, cols, true, &full, "attn_output");
    std::swap(keep, m->allocs);  // `keep` now holds the full matrix's buffers
    m->weight_bytes = before;
    if (!st) {
        w->type = OVF_TYPE_Q8_0;
        w->rows = rows;
        w->cols = cn;
        st = dalloc(m->allocs, (void **)&w->data, (size_t)(rows * cn));
        if (!st) st = dalloc(m->allocs, (void **)&w->scales, (size_t)(rows * cn / 32 * 4));
        if (!st)
            st = cuda_status(cudaMemcpy2D(w->data, (size_t)cn, full.data + c0, (size_t)cols, (size_t)cn, (size_t)rows,
                                          cudaMemcpyDeviceToDevice),
                             "attn_output slice");
        if (!st)
            st = cuda_status(cudaMemcpy2D(w->scales, (size_t)(cn / 32 * 4), full.scales + c0 / 32, (size_t)(cols / 32 * 4),
                                          (size_t)(cn / 32 * 4), (size_t)rows, cudaMemcpyDeviceToDevice),
                             "attn_output scales slice");
        m->weight_bytes += rows * cn + rows * cn / 8;
    }
    for (void *q : keep) cudaFree(q);
    return st;
}

ovf_status fill_rope_tables(ovf_session *s) {
    // Rope/RopeTable.cs:109-133: freq_i = 1/theta^(2i/hd), angle = pos*freq.
    const int hd = s->m->cfg.head_dim, half = hd / 2;
    std::vector<float> c((size_t)s->max_ctx * half), sn((size_t)s->max_ctx * half);
    for (int i = 0; i < half; ++i) {
        volatile float e = 2.0f * (float)i;
        e = e / (float)hd;
        const float freq = 1.0f / powf(s->m->cfg.rope_theta, e);
        for (int p = 0; p < s->max_ctx; ++p) {
            volatile float angle = (float)p * freq;
            c[(size_t)p * half + i] = cosf(angle);
            sn[(size_t)p * half + i] = sinf(angle);
        }
    }
    OVF_CUDA_TRY(cudaMemcpy(s->rope_cos, c.data(), c.size() * 4, cudaMemcpyHostToDevice));
    OVF_CUDA_TRY(cudaMemcpy(s->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
    return OVF_OK;
}

// OVF_EAGER=1 launches the step's kernels directly instead of replaying a
// CUDA graph (profiling and debugging); OVF_NO_PDL=1 drops programmatic
// dependent launch; OVF_NO_L2_PREFETCH=1 drops the L2 prefetch of upcoming
// weights.
bool env_flag(const char *name) {
    const char *v = getenv(name);
    return v && v[0] == '1';
}

int l2_prefetch_mode() {
    static const int mode = [] {
        const char *v = getenv("OVF_L2_PF");
        return v ? atoi(v) : 0;
    }();
    return mode;
}

// Adds a resident weight's bytes (quants, then Q8_0 scales) to an L2
// prefetch list.
void add_prefetch(L2Prefetch &pf, const DevWeight &w) {
    if (!w.data) return;
    int64_t qb = 0;
    if (w.type == OVF_TYPE_Q4_K) qb = w.rows * w.cols / 256 * 144;
    else if (w.type == OVF_TYPE_Q6_K) qb = w.rows * w.cols / 256 * 210;
    else if (w.type == OVF_TYPE_Q8_0) qb = w.rows * w.cols;
    if (qb > 0 && pf.n < 4) {
        pf.ptr[pf.n] = w.data;
        pf.bytes[pf.n++] = qb;
    }
    if (w.type == OVF_TYPE_Q8_0 && w.scales && pf.n < 4) {
        pf.ptr[pf.n] = w.scales;
        pf.bytes[pf.n++] = w.rows * w.cols / 32 * 4;
    }
}

GemvSeg seg_of(const DevWeight &w, const float *bias, float *out) {
    return GemvSeg{w.data, w.scales, bias, out, w.type, (int)w.rows, 0};
}

bool is_kq(int t) { return t == OVF_TYPE_Q4_K || t == OVF_TYPE_Q6_K; }

// OVF_PROFILE_STEP=1 (with OVF_EAGER=1): events after every launch of a
// step, summed per kernel role and printed when the session is destroyed.
struct StepProfiler {
    bool on = false;
    cudaEvent_t last = nullptr;
    std::vector<std::pair<std::string, std::pair<double, int>>> acc;
    std::vector<std::pair<std::string, cudaEvent_t>> pending;
};
static StepProfiler g_prof;

static void prof_mark(cudaStream_t st, const char *label) {
    if (!g_prof.on) return;
    cudaEvent_t e;
    cudaEventCreate(&e);
    cudaEventRecord(e, st);
    g_prof.pending.push_back({label, e});
}

static void prof_flush(cudaStream_t st) {
    if (!g_prof.on || g_prof.pending.empty()) return;
    cudaStreamSynchronize(st);
    for (auto &pe : g_prof.pending) {
        if (g_prof.last) {
            float ms = 0;
            cudaEventElapsedTime(&ms, g_prof.last, pe.second);
            bool found = false;
            for (auto &a : g_prof.acc)
                if (a.first == pe.first) {
                    a.second.first += ms;
                    a.second.second += 1;
                    found = true;
                }
            if (!found) g_prof.acc.push_back({pe.first, {ms, 1}});
            cudaEventDestroy(g_prof.last);
        }
        g_prof.last = pe.second;
    }
    g_prof.pending.clear();
}

static void prof_report() {
    if (!g_prof.on) return;
    for (auto &a : g_prof.acc)
        fprintf(stderr, "[ovf profile] %-8s %8d launches %10.1f us total %8.2f us/launch\n", a.first.c_str(),
                a.second.second, a.second.first * 1e3, a.second.first * 1e3 / a.second.second);
    g_prof.acc.clear();
}

// OVF_TRACE=1: the last step's timeline, per launch role: mean duration
// (first CTA start to last exit), mean time spent before griddepcontrol.wait
// returned, and mean gap / overlap with the previous launch's end.
static void trace_report(ovf_session *s) {
    if (!s->trace || s->trace_n == 0) return;
    std::vector<TraceSlot> t(s->trace_n);
    if (cudaMemcpy(t.data(), s->trace, t.size() * sizeof(TraceSlot), cudaMemcpyDeviceToHost) != cudaSuccess) return;
    struct Acc { double dur = 0, wait = 0, gap = 0, tiles = 0; int n = 0; };
    std::vector<std::pair<std::string, Acc>> acc;
    const unsigned long long t0 = ~t[0].start_c;
    unsigned long long prev_end = t0;
    for (int i = 0; i < s->trace_n; ++i) {
        const unsigned long long st = ~t[i].start_c, en = t[i].end, wt = t[i].waited;
        Acc *a = nullptr;
        for (auto &x : acc)
            if (x.first == s->trace_labels[i]) a = &x.second;
        if (!a) {
            acc.push_back({s->trace_labels[i], Acc{}});
            a = &acc.back().second;
        }
        a->dur += (double)(en - st) / 1e3;
        a->wait += wt > st ? (double)(wt - st) / 1e3 : 0.0;
        a->gap += ((double)st - (double)prev_end) / 1e3;
        a->tiles += t[i].tiles > wt && wt > 0 ? (double)(t[i].tiles - wt) / 1e3 : 0.0;
        a->n += 1;
        prev_end = en;
    }
    fprintf(stderr, "[ovf trace] step span %.1f us over %d launches\n", (double)(prev_end - t0) / 1e3, s->trace_n);
    for (auto &x : acc)
        fprintf(stderr,
                "[ovf trace] %-8s n=%3d  dur %8.2f us  pre-wait %7.2f us  start-after-prev-end %7.2f us  "
                "tiles-done-after-wait %7.2f us\n",
                x.first.c_str(), x.second.n, x.second.dur / x.second.n, x.second.wait / x.second.n,
                x.second.gap / x.second.n, x.second.tiles / x.second.n);
}

// Tensor parallelism: the exchange slot `slot` of the model's arena.
TpExchange tp_exchange(const ovf_model *m, int slot) {
    TpExchange x{};
    for (int w = 0; w < m->tp_world; ++w) x.flags_peer[w] = reinterpret_cast<unsigned *>(m->peer[w] + m->off_flags);
    x.flags_own = reinterpret_cast<const unsigned *>(m->arena + m->off_flags);
    x.epoch = reinterpret_cast<const unsigned *>(m->arena + m->off_epoch);
    x.world = m->tp_world;
    x.rank = m->tp_rank;
    x.slot = slot;
    return x;
}

// Every rank's exchange buffer at byte offset `off` + `elem` floats.
void tp_dsts(const ovf_model *m, size_t off, size_t elem, GemvParams *p) {
    for (int w = 0; w < m->tp_world; ++w) p->tp_dst[w] = reinterpret_cast<float *>(m->peer[w] + off) + elem;
    p->tp_world = m->tp_world;
    p->tp_rank = m->tp_rank;
}

// MoE FFN of one decode token (MoeFeedForwardBlock.Decode, :79-138): the
// router on the device, then for each of the k selected experts a fused
// gate/up GEMV (SiLU*up) and a down GEMV whose weights are picked by the
// expert index the router left in device memory (no host round trip, so the
// step stays one CUDA graph), then the weighted sum in top-k order, the
// residual, and the next RMSNorm's scale.
template <class Slot>
ovf_status enqueue_moe_ffn(ovf_session *s, const DevLayer &L, cudaStream_t st, Slot tslot) {
    const ovf_model_config &c = s->m->cfg;
    const int D = c.d_model, FF = c.d_ff, K = c.n_experts_used;
    ovf_status r = launch_moe_route(s->after, D, L.ffn_norm, &s->norm_s[1], L.router, 1, D, c.n_experts, K,
                                    c.normalize_experts, s->msel, s->mw, st, true);
    if (r) return r;
    const ovf_model *m = s->m;
    const bool ep = m->tp_world > 1;
    const int l = (int)(&L - m->layers.data());
    for (int j = 0; j < K; ++j) {
        GemvParams p{};
        p.nseg = 2;
        p.pair = 1;
        if (ep) {
            p.expert_mod = m->tp_world;
            p.expert_rank = m->tp_rank;
        }
        p.seg[0] = seg_of(L.gate, nullptr, s->mh + (size_t)j * FF);
        p.seg[1] = seg_of(L.up, nullptr, s->mh + (size_t)j * FF);
        p.seg[0].rows = p.seg[1].rows = FF;
        p.K = D;
        p.act_mode = ACT_F32_RMSNORM;
        p.x = s->after;
        p.gamma = L.ffn_norm;
        p.norm_scale = &s->norm_s[1];
        p.eps = c.eps;
        p.epi = EPI_SILU_PAIR;
        p.expert_sel = s->msel;
        p.expert_slot = j;
        p.expert_wstride = L.gu_wstride;
        p.expert_sstride = L.gu_sstride;
        p.trace = tslot("gateup");
        if ((r = gemv_launch(p, st, true))) return r;
        GemvParams q{};
        q.nseg = 1;
        q.seg[0] = seg_of(L.down, nullptr, s->meo + (size_t)j * D);
        q.seg[0].rows = D;
        q.K = FF;
        q.act_mode = ACT_F32;
        q.x = s->mh + (size_t)j * FF;
        q.epi = EPI_STORE;
        q.expert_sel = s->msel;
        q.expert_slot = j;
        q.expert_wstride = L.d_wstride;
        q.expert_sstride = L.d_sstride;
        if (ep) {
            // the owner of expert sel[j] writes its output into every rank's slot j
            q.expert_mod = m->tp_world;
            q.expert_rank = m->tp_rank;
            q.epi = EPI_ROWS_TP;
            tp_dsts(m, m->off_moe, ((size_t)l * K) * D, &q);
            q.tp_index0 = j;
            q.tp_rows = D;
        }
        q.trace = tslot("down");
        if ((r = gemv_launch(q, st, true))) return r;
    }
    if (ep) {
        const float *recv = reinterpret_cast<const float *>(m->arena + m->off_moe) + (size_t)l * K * D;
        return launch_tp_moe_combine(tp_exchange(m, 2 * l + 1), recv, s->mw, K, s->after, s->hidden, &s->norm_s[0], D,
                                     c.eps, st, true);
    }
    return launch_moe_combine(s->after, s->meo, s->mw, K, D, s->hidden, &s->norm_s[0], c.eps, st, true);
}

// Enqueues one token's kernels on s->stream.
ovf_status enqueue_step(ovf_session *s, bool with_logits) {
    ovf_model *m = s->m;
    const ovf_model_config &c = m->cfg;
    const cudaStream_t st = s->stream;
    const bool tp = m->tp_world > 1;
    // this rank's heads (all of them on one GPU)
    const int D = c.d_model, H = m->h_loc, KVH = m->kvh_loc, hd = c.head_dim;
    s->trace_n = 0;
    auto tslot = [&](const char *label) -> TraceSlot * {
        if (!s->trace || s->trace_n >= s->trace_cap) return nullptr;
        if ((int)s->trace_labels.size() <= s->trace_n) s->trace_labels.push_back(label);
        return &s->trace[s->trace_n++];
    };
    if (s->trace) OVF_CUDA_TRY(cudaMemsetAsync(s->trace, 0, (size_t)s->trace_cap * sizeof(TraceSlot), st));
    ovf_status r = launch_embed(s->step, m->embed.type, m->embed.data, m->embed.scales, D, s->hidden, s->step,
                                &s->norm_s[0], c.eps, tslot("embed"), st, true,
                                tp ? reinterpret_cast<unsigned *>(m->arena + m->off_epoch) : nullptr);
    prof_mark(st, "embed");
    if (r) return r;
    for (int l = 0; l < c.n_layers; ++l) {
        const DevLayer &L = m->layers[l];
        // Q/K/V: one launch when the three share an activation format.
        const bool kq = is_kq(L.wq.type);
        const bool same_family = is_kq(L.wk.type) == kq && is_kq(L.wv.type) == kq;
        if (same_family) {
            GemvParams p{};
            p.nseg = 3;
            p.seg[0] = seg_of(L.wq, L.bq, s->q);
            p.seg[1] = seg_of(L.wk, L.bk, s->k);
            p.seg[2] = seg_of(L.wv, L.bv, s->v);
            p.K = D;
            p.act_mode = ACT_F32_RMSNORM;
            p.x = s->hidden;
            p.gamma = L.attn_norm;
            p.norm_scale = &s->norm_s[0];
            p.eps = c.eps;
            p.epi = EPI_STORE;
            p.fill_sentinel = tp ? nullptr : s->after;  // Wo's norm CTA watches `after` being written
            p.fill_n = D;
            p.trace = tslot("qkv");
            if ((r = gemv_launch(p, st, true))) return r;
            prof_mark(st, "qkv");
        } else {
            const DevWeight *ws[3] = {&L.wq, &L.wk, &L.wv};
            const float *bs[3] = {L.bq, L.bk, L.bv};
            float *os[3] = {s->q, s->k, s->v};
            for (int i = 0; i < 3; ++i) {
                GemvParams p{};
                p.nseg = 1;
                p.seg[0] = seg_of(*ws[i], bs[i], os[i]);
                p.K = D;
                p.act_mode = ACT_F32_RMSNORM;
                p.x = s->hidden;
                p.gamma = L.attn_norm;
                p.norm_scale = &s->norm_s[0];
                p.eps = c.eps;
                p.epi = EPI_STORE;
                if (i == 0 && !tp) {
                    p.fill_sentinel = s->after;
                    p.fill_n = D;
                }
                p.trace = tslot("qkv");
                if ((r = gemv_launch(p, st, true))) return r;
                prof_mark(st, "qkv");
            }
        }
        AttnParams a{};
        a.q = s->q;
        a.k_new = s->k;
        a.v_new = s->v;
        const size_t esz = s->kv_dtype == OVF_KV_F32 ? 4 : s->kv_dtype == OVF_KV_Q8 ? 1 : 2;
        a.kc = (__half *)((char *)s->kc + (size_t)l * KVH * s->max_ctx * hd * esz);
        a.vc = (__half *)((char *)s->vc + (size_t)l * KVH * s->max_ctx * hd * esz);
        if (s->kv_dtype == OVF_KV_Q8) {
            a.ks = s->ks + (size_t)l * KVH * s->max_ctx;
            a.vs = s->vs + (size_t)l * KVH * s->max_ctx;
        }
        a.out = s->attn;
        a.rope_cos = s->rope_cos;
        a.rope_sin = s->rope_sin;
        a.pos_dev = &s->step->cur_pos;
        a.partial = s->partial;
        a.counters = s->counters;
        a.split_half = c.rope_split_half;
        a.H = H;
        a.KVH = KVH;
        a.hd = hd;
        a.max_ctx = s->max_ctx;
        a.scale = 1.0f / sqrtf((float)hd);
        if (l2_prefetch_mode() & 1) add_prefetch(a.pf, L.wo);
        if (l2_prefetch_mode() & 2) {
            add_prefetch(a.pf, L.gate);
            add_prefetch(a.pf, L.up);
        }
        a.trace = tslot("attn");
        a.no_kv_prefetch = env_flag("OVF_ATTN_NOPF") ? 1 : 0;
        if ((r = launch_attention_exact(a, s->max_ctx, st, true, s->kv_dtype))) return r;
        prof_mark(st, "attn");
        {
            // Wo: per-head Q8_0 (G = hd/32 blocks per head), heads summed in
            // ascending order on top of the bias, then the residual.
            GemvParams p{};
            p.nseg = 1;
            p.seg[0] = seg_of(L.wo, L.bo, s->after);
            p.K = H * hd;
            p.q8_group = hd / 32;
            p.act_mode = ACT_F32;
            p.x = s->attn;
            if (tp) {
                // this rank's heads' outputs into every rank's exchange buffer
                p.seg[0].bias = nullptr;
                p.epi = EPI_GROUPS_TP;
                tp_dsts(m, m->off_heads, (size_t)l * c.n_heads * D, &p);
                p.tp_index0 = m->tp_rank * H;
                p.tp_rows = D;
            } else {
                p.epi = EPI_RESIDUAL;
                p.resid = s->hidden;
                p.norm_out = &s->norm_s[1];  // RMSNorm scale of `after` for the FFN
            }
            if (l2_prefetch_mode() & 4) add_prefetch(p.pf, L.down);
            p.eps = c.eps;
            p.trace = tslot("wo");
            if ((r = gemv_launch(p, st, true))) return r;
            if (tp) {
                // after = hidden + (((bias + y_0) + y_1) + ...), every head in order
                const float *recv = reinterpret_cast<const float *>(m->arena + m->off_heads) + (size_t)l * c.n_heads * D;
                if ((r = launch_tp_sum_combine(tp_exchange(m, 2 * l), recv, c.n_heads, L.bo, s->hidden, s->after,
                                               &s->norm_s[1], D, c.eps, st, true)))
                    return r;
            }
            prof_mark(st, "wo");
        }
        if (c.n_experts > 0) {
            if ((r = enqueue_moe_ffn(s, L, st, tslot))) return r;
            continue;
        }
        if (L.gate.type == L.up.type) {
            GemvParams p{};
            p.nseg = 2;
            p.pair = 1;
            p.seg[0] = seg_of(L.gate, nullptr, s->h);
            p.seg[1] = seg_of(L.up, nullptr, s->h);
            p.K = D;
            p.act_mode = ACT_F32_RMSNORM;
            p.x = s->after;
            p.gamma = L.ffn_norm;
            p.norm_scale = &s->norm_s[1];
            p.eps = c.eps;
            p.epi = EPI_SILU_PAIR;
            p.fill_sentinel = tp ? nullptr : s->hidden;  // the down projection's norm CTA watches `hidden`
            p.fill_n = D;
            if ((l2_prefetch_mode() & 8) && l + 1 < c.n_layers) {
                const DevLayer &N = m->layers[l + 1];
                add_prefetch(p.pf, N.wq);
                add_prefetch(p.pf, N.wk);
                add_prefetch(p.pf, N.wv);
            }
            p.trace = tslot("gateup");
            if ((r = gemv_launch(p, st, true))) return r;
            prof_mark(st, "gateup");
        } else {
            const DevWeight *ws[2] = {&L.gate, &L.up};
            float *os[2] = {s->gtmp, s->utmp};
            for (int i = 0; i < 2; ++i) {
                GemvParams p{};
                p.nseg = 1;
                p.seg[0] = seg_of(*ws[i], nullptr, os[i]);
                p.K = D;
                p.act_mode = ACT_F32_RMSNORM;
                p.x = s->after;
                p.gamma = L.ffn_norm;
                p.norm_scale = &s->norm_s[1];
                p.eps = c.eps;
                p.epi = EPI_STORE;
                if (i == 0 && !tp) {
                    p.fill_sentinel = s->hidden;
                    p.fill_n = D;
                }
                p.trace = tslot("gateup");
                if ((r = gemv_launch(p, st, true))) return r;
                prof_mark(st, "gateup");
            }
            if ((r = launch_silu_mul(s->gtmp, s->utmp, s->h, m->ff_loc, st, true))) return r;
            prof_mark(st, "gateup");
        }
        {
            GemvParams p{};
            p.nseg = 1;
            p.seg[0] = seg_of(L.down, nullptr, s->hidden);
            p.K = m->ff_loc;
            p.act_mode = ACT_F32;
            p.x = s->h;
            if (tp) {
                // this rank's block terms of every row into every rank's buffer
                p.epi = EPI_TERMS_TP;
                tp_dsts(m, m->off_terms, (size_t)l * m->nb_down * D, &p);
                p.tp_index0 = m->tp_rank * (m->nb_down / m->tp_world);
                p.tp_rows = D;
            } else {
                p.epi = EPI_RESIDUAL;
                p.resid = s->after;
                p.norm_out = &s->norm_s[0];  // RMSNorm scale of the new hidden: next layer / final norm
            }
            p.eps = c.eps;
            p.trace = tslot("down");
            if ((r = gemv_launch(p, st, true))) return r;
            if (tp) {
                // hidden = after + (((0 + t_0) + t_1) + ...), every block in order
                const float *recv = reinterpret_cast<const float *>(m->arena + m->off_terms) + (size_t)l * m->nb_down * D;
                if ((r = launch_tp_sum_combine(tp_exchange(m, 2 * l + 1), recv, m->nb_down, nullptr, s->after,
                                               s->hidden, &s->norm_s[0], D, c.eps, st, true)))
                    return r;
            }
            prof_mark(st, "down");
        }
    }
    if (with_logits) {
        GemvParams p{};
        p.nseg = 1;
        p.seg[0] = seg_of(m->lm_head, nullptr, s->logits);
        p.K = D;
        p.act_mode = ACT_F32_RMSNORM;
        p.x = s->hidden;
        p.gamma = m->final_norm;
        p.norm_scale = &s->norm_s[0];
        p.eps = c.eps;
        p.epi = EPI_LOGITS_ARGMAX;
        p.step = s->step;
        p.tokens_out = s->tokens_log;
        if (tp) {
            // this rank's vocabulary rows into every rank's logits, keys published
            p.epi = EPI_LOGITS_TP;
            tp_dsts(m, m->off_logits, 0, &p);
            for (int w = 0; w < m->tp_world; ++w)
                p.tp_keys[w] = reinterpret_cast<unsigned long long *>(m->peer[w] + m->off_keys);
            p.tp_index0 = m->tp_rank * m->v_loc;
        }
        p.trace = tslot("lmhead");
        if ((r = gemv_launch(p, st, true))) return r;
        if (tp) {
            if ((r = launch_tp_lm_finish(tp_exchange(m, 2 * c.n_layers),
                                         reinterpret_cast<const unsigned long long *>(m->arena + m->off_keys), s->step,
                                         s->tokens_log, st, true)))
                return r;
            OVF_CUDA_TRY(cudaMemcpyAsync(s->logits, m->arena + m->off_logits, (size_t)c.vocab * 4,
                                         cudaMemcpyDeviceToDevice, st));
        }
        prof_mark(st, "lmhead");
    }
    return OVF_OK;
}

ovf_status capture(ovf_session *s, bool with_logits, cudaGraphExec_t *out) {
    cudaGraph_t g = nullptr;
    OVF_CUDA_TRY(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
    ovf_status r = enqueue_step(s, with_logits);
    cudaError_t e = cudaStreamEndCapture(s->stream, &g);
    if (r) {
        if (g) cudaGraphDestroy(g);
        return r;
    }
    if (e != cudaSuccess) return cuda_status(e, "cudaStreamEndCapture");
    e = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    return cuda_status(e, "cudaGraphInstantiate");
}


ovf_status run_step(ovf_session *s, bool with_logits) {
    cudaGraphExec_t *gx = with_logits ? &s->graph_logits : &s->graph_nologits;
    if (env_flag("OVF_EAGER")) {
        g_prof.on = env_flag("OVF_PROFILE_STEP");
        if (g_prof.on && !g_prof.last) {
            cudaEventCreate(&g_prof.last);
            cudaEventRecord(g_prof.last, s->stream);
        }
        ovf_status r = enqueue_step(s, with_logits);
        prof_flush(s->stream);
        if (r) return r;
        s->pos += 1;
        if (with_logits) s->n_logits += 1;
        return OVF_OK;
    }
    if (!*gx) {
        ovf_status r = capture(s, with_logits, gx);
        if (r) return r;
    }
    OVF_CUDA_TRY(cudaGraphLaunch(*gx, s->stream));
    s->pos += 1;
    if (with_logits) s->n_logits += 1;
    return OVF_OK;
}

// ------------------------------------------------------- batched prefill
// CachedLlamaSession.PrefillBatchedQuant (:818-835) with
// CachedTransformerBlock.DecodeBatchedQuant (:388-478): the prompt runs
// through each layer as a chunk of rows — RMSNorm per row, the
// weight-stationary projections (each weight tile read once per chunk),
// attention per row in position order (the row's key and value appended
// before it attends, causal over [0, pos]), Wo with head-ordered sums and
// the residual, the FFN the same way — and only the last row is projected
// to logits.  Every row's arithmetic is the single-token step's, so the
// session ends in the state n decode steps would leave, bit for bit.
constexpr int kPrefillRows = 256;       // rows per chunk
constexpr int kPrefillThreshold = 16;   // BatchedPrefillThreshold (CachedLlamaSession.cs:805)

ovf_status prefill_alloc(ovf_session *s) {
    if (s->pf_rows) return OVF_OK;
    const ovf_model_config &c = s->m->cfg;
    const size_t R = kPrefillRows, D = c.d_model, QD = (size_t)c.n_heads * c.head_dim,
                 KD = (size_t)c.n_kv_heads * c.head_dim, FF = c.d_ff;
    const size_t KM = std::max(std::max(D, QD), FF);
    ovf_status st = OVF_OK;
    auto A = [&](void **p, size_t bytes) {
        if (!st) st = dalloc(s->allocs, p, bytes);
    };
    A((void **)&s->px, R * D * 4);
    A((void **)&s->pa, R * D * 4);
    A((void **)&s->pn, R * D * 4);
    A((void **)&s->pq, R * QD * 4);
    A((void **)&s->pk, R * KD * 4);
    A((void **)&s->pv, R * KD * 4);
    A((void **)&s->patt, R * QD * 4);
    A((void **)&s->pg, R * FF * 4);
    A((void **)&s->pu, R * FF * 4);
    A((void **)&s->ph, R * FF * 4);
    A((void **)&s->paq, R * KM);
    A((void **)&s->pas, R * KM / 32 * 4);
    A((void **)&s->pab, R * KM / 16 * 2);
    A(&s->ptc, (size_t)std::max(tc_scratch_bytes((int64_t)R, (int64_t)KM), tc8_scratch_bytes((int64_t)R, (int64_t)KM)));
    A((void **)&s->ptok, (size_t)(s->max_ctx + 1) * 4);
    A((void **)&s->pscale, 16);
    if (!st && c.n_experts > 0) st = moe_rows_alloc(c, kPrefillRows, s->allocs, &s->pmoe);
    const int64_t pfl = attn_rows_scratch_floats(kPrefillRows, s->m->h_loc, s->max_ctx);
    if (!st && attn_rows_supported(c.head_dim, s->kv_dtype) && pfl * 4 <= ((int64_t)512 << 20))
        A((void **)&s->pattn, (size_t)pfl * 4);
    if (!st) s->pf_rows = kPrefillRows;
    return st;
}

// Activation rows of `x` quantized for weight `w` (Q8_K for K-quants, Q8_0
// otherwise), unless they already are (`*fam`: 1 = Q8_K, 2 = Q8_0).
struct ActRows {  // quantized activation rows (Q8_K or Q8_0) of a batch
    int8_t *aq;
    float *as;
    int16_t *ab;
    void *tc = nullptr;  // tensor-core operand scratch (tc_scratch_bytes of the rows), or none
};

// From this many rows on, Q4_K, Q6_K and Q8_0 projections run on the tensor
// cores (tc_q4k_project_kernel, tc_q6k_project_kernel, tc_q80_project_kernel); fewer rows stay on the dp4a
// weight-stationary kernel, which streams the weights once with no operand
// expansion.  All are bit-identical to the reference's per-row dot.
constexpr int kTcMinRows = 32;

ovf_status quantize_rows_for(const ActRows &ar, const DevWeight &w, const float *x, int rows, int64_t k, int *fam,
                             cudaStream_t st) {
    const int want = is_kq(w.type) ? 1 : 2;
    if (*fam == want) return OVF_OK;
    *fam = want;
    return want == 1 ? launch_quantize_q8k(x, rows * k, ar.aq, ar.as, ar.ab, st)
                     : launch_quantize_q8_0(x, rows * k, ar.aq, ar.as, st);
}

ovf_status project_rows(const ActRows &ar, const DevWeight &w, const float *bias, float *y, int rows, cudaStream_t st,
                        int group = 0, const float *resid = nullptr) {
    if (ar.tc && group == 0 && rows >= kTcMinRows && tc_project_supported(w.type, w.rows, w.cols, rows))
        return launch_tc_project(w.type, w.data, bias, ar.aq, ar.as, ar.ab, y, w.rows, w.cols, rows, ar.tc, st, resid);
    if (ar.tc && w.type == OVF_TYPE_Q6_K && group == 0 && rows >= kTcMinRows && tc6_project_supported(w.rows, w.cols, rows))
        return launch_tc6_project(w.data, bias, ar.aq, ar.as, ar.ab, y, w.rows, w.cols, rows, ar.tc, st, resid);
    if (ar.tc && w.type == OVF_TYPE_Q8_0 && rows >= kTcMinRows && tc8_project_supported(w.rows, w.cols, rows, group))
        return launch_tc8_project(reinterpret_cast<const int8_t *>(w.data), w.scales, bias, ar.aq, ar.as, y, w.rows, w.cols,
                                  rows, group, ar.tc, st, resid);
    const size_t qbytes = w.type == OVF_TYPE_Q8_0 ? (size_t)w.rows * w.cols : (size_t)tensor_bytes(w.type, w.rows, w.cols);
    return launch_batched_project(w.type, w.data, w.scales, qbytes, bias, ar.aq, ar.as, ar.ab, y, w.rows, w.cols,
                                  rows, st, group, resid);
}


// Row buffers of one batch of hidden states ([rows][width] each).
struct RowBufs {
    ActRows ar;
    float *x, *a, *n, *q, *k, *v, *att, *g, *u, *h;
};

// RMSNorm of x (attn_norm) -> n, then Q/K/V of every row (with biases).
ovf_status rows_norm_qkv(const ovf_model *m, const DevLayer &L, const RowBufs &b, int M, cudaStream_t st) {
    const ovf_model_config &c = m->cfg;
    const int D = c.d_model;
    int fam = 0;
    ovf_status r;
    if ((r = launch_rmsnorm_rows(b.x, L.attn_norm, b.n, M, D, c.eps, nullptr, st))) return r;
    if ((r = quantize_rows_for(b.ar, L.wq, b.n, M, D, &fam, st))) return r;
    if ((r = project_rows(b.ar, L.wq, L.bq, b.q, M, st))) return r;
    if ((r = quantize_rows_for(b.ar, L.wk, b.n, M, D, &fam, st))) return r;
    if ((r = project_rows(b.ar, L.wk, L.bk, b.k, M, st))) return r;
    if ((r = quantize_rows_for(b.ar, L.wv, b.n, M, D, &fam, st))) return r;
    return project_rows(b.ar, L.wv, L.bv, b.v, M, st);
}

// Wo (Q8_0, heads in order on the bias) + residual x -> a; RMSNorm(a) ->
// n; gate/up; SiLU*up -> h; down + residual a -> x.
// SwiGLU of rows x ([M][D], normalized) through gate/up/down -> y ([M][D]),
// optionally + resid.
ovf_status rows_swiglu(const DevWeight &gate, const DevWeight &up, const DevWeight &down, const RowBufs &b,
                       const float *x, float *y, const float *resid, int M, int D, int FF, cudaStream_t st) {
    int fam = 0;
    ovf_status r;
    if ((r = quantize_rows_for(b.ar, gate, x, M, D, &fam, st))) return r;
    if ((r = project_rows(b.ar, gate, nullptr, b.g, M, st))) return r;
    if ((r = quantize_rows_for(b.ar, up, x, M, D, &fam, st))) return r;
    if ((r = project_rows(b.ar, up, nullptr, b.u, M, st))) return r;
    if ((r = launch_silu_mul(b.g, b.u, b.h, (int64_t)M * FF, st, false))) return r;
    fam = 0;
    if ((r = quantize_rows_for(b.ar, down, b.h, M, FF, &fam, st))) return r;
    return project_rows(b.ar, down, nullptr, y, M, st, 0, resid);
}

// The FFN of M rows: b.a holds the residual stream after attention, b.n its
// RMSNorm; the result (+ residual) lands in b.x.  Dense: one SwiGLU.  MoE
// (MoeFeedForwardBlock.DecodeBatched, :140-243): route every row, group the
// rows per expert (host round trip for the counts), run each used expert's
// SwiGLU once over its rows, stash each output at the row's top-k slot and
// sum the slots in top-k order, so every row equals a single-token decode.
ovf_status rows_ffn(const ovf_model *m, const DevLayer &L, const RowBufs &b, MoeRows *mr, int M, cudaStream_t st) {
    const ovf_model_config &c = m->cfg;
    const int D = c.d_model, FF = c.d_ff;
    if (c.n_experts == 0) return rows_swiglu(L.gate, L.up, L.down, b, b.n, b.x, b.a, M, D, FF, st);
    const int E = c.n_experts, K = c.n_experts_used, R = mr->cap;
    ovf_status r;
    if ((r = launch_moe_route(b.n, D, nullptr, nullptr, L.router, M, D, E, K, c.normalize_experts, mr->sel, mr->w, st,
                              false)))
        return r;
    int32_t *hsel = mr->host, *hrows = mr->host + (size_t)R * K, *hslots = hrows + (size_t)E * R;
    OVF_CUDA_TRY(cudaMemcpyAsync(hsel, mr->sel, (size_t)M * K * 4, cudaMemcpyDeviceToHost, st));
    OVF_CUDA_TRY(cudaStreamSynchronize(st));
    std::vector<int> count(E, 0);
    for (int e = 0; e < E; ++e)
        for (int n = 0; n < M; ++n)
            for (int j = 0; j < K; ++j)
                if (hsel[(size_t)n * K + j] == e) {
                    hrows[(size_t)e * R + count[e]] = n;
                    hslots[(size_t)e * R + count[e]] = j;
                    ++count[e];
                    break;
                }
    OVF_CUDA_TRY(cudaMemcpyAsync(mr->idx, hrows, (size_t)2 * E * R * 4, cudaMemcpyHostToDevice, st));
    for (int e = 0; e < E; ++e) {
        if (!count[e]) continue;
        const int32_t *rows = mr->idx + (size_t)e * R, *slots = mr->idx + (size_t)E * R + (size_t)e * R;
        if ((r = launch_gather_rows(b.n, rows, count[e], D, mr->gx, st))) return r;
        if ((r = rows_swiglu(expert_view(L.gate, FF, e), expert_view(L.up, FF, e), expert_view(L.down, D, e), b, mr->gx,
                             mr->eo, nullptr, count[e], D, FF, st)))
            return r;
        if ((r = launch_scatter_slots(mr->eo, rows, slots, count[e], K, D, mr->slot, st))) return r;
    }
    return launch_moe_combine_rows(b.a, mr->slot, mr->w, K, M, D, b.x, st);
}

ovf_status rows_wo_ffn(const ovf_model *m, const DevLayer &L, const RowBufs &b, MoeRows *mr, int M, cudaStream_t st) {
    const ovf_model_config &c = m->cfg;
    const int D = c.d_model, QD = c.n_heads * c.head_dim, hd = c.head_dim;
    int fam = 0;
    ovf_status r;
    if ((r = quantize_rows_for(b.ar, L.wo, b.att, M, QD, &fam, st))) return r;
    const int g = hd / 32 < QD / 32 ? hd / 32 : 0;
    if ((r = project_rows(b.ar, L.wo, L.bo, b.a, M, st, g, b.x))) return r;
    if ((r = launch_rmsnorm_rows(b.a, L.ffn_norm, b.n, M, D, c.eps, nullptr, st))) return r;
    return rows_ffn(m, L, b, mr, M, st);
}

// Enqueues the batched prefill of tokens [0, n) (already in s->ptok) at
// positions s->pos ..; the last row's logits and argmax land where a decode
// step's would.
ovf_status enqueue_prefill_batched(ovf_session *s, int n, bool all_rows = false) {
    ovf_model *m = s->m;
    const ovf_model_config &c = m->cfg;
    const cudaStream_t st = s->stream;
    const int D = c.d_model, H = c.n_heads, KVH = c.n_kv_heads, hd = c.head_dim, FF = c.d_ff;
    const int QD = H * hd, KD = KVH * hd;
    const int base = s->pos;
    const ActRows ar{s->paq, s->pas, s->pab, s->ptc};
    const RowBufs pb{ar, s->px, s->pa, s->pn, s->pq, s->pk, s->pv, s->patt, s->pg, s->pu, s->ph};
    ovf_status r = OVF_OK;
    int last_rows = 0;
    for (int r0 = 0; r0 < n; r0 += s->pf_rows) {
        const int M = std::min(s->pf_rows, n - r0);
        last_rows = M;
        if ((r = launch_embed_rows(s->ptok + r0, M, m->embed.type, m->embed.data, m->embed.scales, D, s->px, st)))
            return r;
        for (int l = 0; l < c.n_layers; ++l) {
            const DevLayer &L = m->layers[l];
            int fam = 0;
            if ((r = launch_rmsnorm_rows(s->px, L.attn_norm, s->pn, M, D, c.eps, nullptr, st))) return r;
            if ((r = quantize_rows_for(ar, L.wq, s->pn, M, D, &fam, st))) return r;
            if ((r = project_rows(ar, L.wq, L.bq, s->pq, M, st))) return r;
            if ((r = quantize_rows_for(ar, L.wk, s->pn, M, D, &fam, st))) return r;
            if ((r = project_rows(ar, L.wk, L.bk, s->pk, M, st))) return r;
            if ((r = quantize_rows_for(ar, L.wv, s->pn, M, D, &fam, st))) return r;
            if ((r = project_rows(ar, L.wv, L.bv, s->pv, M, st))) return r;
            const size_t esz = s->kv_dtype == OVF_KV_F32 ? 4 : s->kv_dtype == OVF_KV_Q8 ? 1 : 2;
            {
                // every row's key and value are appended first, then one launch
                // attends all rows (each causal at its own position)
                AttnParams a{};
                a.q = s->pq;
                a.rows = M;
                a.kc = (__half *)((char *)s->kc + (size_t)l * KVH * s->max_ctx * hd * esz);
                a.vc = (__half *)((char *)s->vc + (size_t)l * KVH * s->max_ctx * hd * esz);
                if (s->kv_dtype == OVF_KV_Q8) {
                    a.ks = s->ks + (size_t)l * KVH * s->max_ctx;
                    a.vs = s->vs + (size_t)l * KVH * s->max_ctx;
                }
                a.out = s->patt;
                a.rope_cos = s->rope_cos;
                a.rope_sin = s->rope_sin;
                a.seq_len_host = base + r0 + 1;
                a.split_half = c.rope_split_half;
                a.H = H;
                a.KVH = KVH;
                a.hd = hd;
                a.max_ctx = s->max_ctx;
                a.scale = 1.0f / sqrtf((float)hd);
                if ((r = launch_kv_append_rows(a, s->pk, s->pv, M, base + r0, s->kv_dtype, st))) return r;
                if (s->pattn) {
                    if ((r = launch_attention_rows(a, base + r0, s->pattn, st, s->kv_dtype))) return r;
                } else if ((r = launch_attention_exact(a, s->max_ctx, st, false, s->kv_dtype))) {
                    return r;
                }
            }
            // Wo (Q8_0) per head, heads in order on the bias, + residual; FFN
            if ((r = rows_wo_ffn(m, L, pb, &s->pmoe, M, st))) return r;
        }
    }
    if (all_rows) {
        // every row of the (single) chunk to logits: final norm per row, the
        // LM head over all rows with one read of its weights, argmax per row
        // (CachedGptStack.ProjectLogitsBatched); the last row's logits and
        // argmax become the session's, as after a decode step
        int fam = 0;
        if ((r = launch_rmsnorm_rows(s->px, m->final_norm, s->pn, n, D, c.eps, nullptr, st))) return r;
        if ((r = quantize_rows_for(ar, m->lm_head, s->pn, n, D, &fam, st))) return r;
        if ((r = project_rows(ar, m->lm_head, nullptr, s->vlogits, n, st))) return r;
        if ((r = launch_argmax_rows(s->vlogits, n, c.vocab, s->vargmax, st))) return r;
        OVF_CUDA_TRY(cudaMemcpyAsync(s->logits, s->vlogits + (size_t)(n - 1) * c.vocab, (size_t)c.vocab * 4,
                                     cudaMemcpyDeviceToDevice, st));
        return launch_batch_finish(s->step, base + n - 1, base + n, s->vargmax + n - 1, s->tokens_log, st);
    }
    // final norm + logits + argmax of the last prompt row
    const float *last = s->px + (size_t)(last_rows - 1) * D;
    if ((r = launch_rmsnorm_rows(last, m->final_norm, s->pn, 1, D, c.eps, s->pscale, st))) return r;
    if ((r = launch_set_step_pos(s->step, base + n - 1, base + n, st))) return r;
    GemvParams p{};
    p.nseg = 1;
    p.seg[0] = seg_of(m->lm_head, nullptr, s->logits);
    p.K = D;
    p.act_mode = ACT_F32_RMSNORM;
    p.x = last;
    p.gamma = m->final_norm;
    p.norm_scale = s->pscale;
    p.eps = c.eps;
    p.epi = EPI_LOGITS_ARGMAX;
    p.step = s->step;
    p.tokens_out = s->tokens_log;
    return gemv_launch(p, st, false);
}

// ------------------------------------------------- multi-session decode
// N sessions of one model decode one token each as rows of one batch:
// embedding rows, RMSNorm rows, the weight-stationary projections (each
// weight tile read once for all N), attention per row on that session's own
// cache at its own position, Wo/FFN rows, final norm, LM head rows and the
// argmax per row.  Every row's arithmetic is its session's decode step, so
// the results equal N single decodes, bit for bit (the reference serves
// concurrent sessions one DecodeToken at a time).
constexpr int kBatchMax = 64;

ovf_status batch_alloc(ovf_model *m) {
    if (m->b_rows) return OVF_OK;
    const ovf_model_config &c = m->cfg;
    const size_t R = kBatchMax, D = c.d_model, QD = (size_t)c.n_heads * c.head_dim,
                 KD = (size_t)c.n_kv_heads * c.head_dim, FF = c.d_ff, V = c.vocab;
    const size_t KM = std::max(std::max(D, QD), FF);
    ovf_status st = OVF_OK;
    auto A = [&](void **p, size_t bytes) {
        if (!st) st = dalloc(m->allocs, p, bytes);
    };
    A((void **)&m->bx, R * D * 4);
    A((void **)&m->ba, R * D * 4);
    A((void **)&m->bn, R * D * 4);
    A((void **)&m->bq, R * QD * 4);
    A((void **)&m->bk, R * KD * 4);
    A((void **)&m->bv, R * KD * 4);
    A((void **)&m->batt, R * QD * 4);
    A((void **)&m->bg, R * FF * 4);
    A((void **)&m->bu, R * FF * 4);
    A((void **)&m->bh, R * FF * 4);
    A((void **)&m->baq, R * KM);
    A((void **)&m->bas, R * KM / 32 * 4);
    A((void **)&m->bab, R * KM / 16 * 2);
    A((void **)&m->blogits, R * V * 4);
    A((void **)&m->btok, R * 4);
    A((void **)&m->bargmax, R * 4);
    if (!st && !m->btok_host) st = cuda_status(cudaMallocHost(&m->btok_host, R * 4), "cudaMallocHost");
    if (!st && c.n_experts > 0) st = moe_rows_alloc(c, kBatchMax, m->allocs, &m->bmoe);
    if (!st) m->b_rows = kBatchMax;
    return st;
}

ovf_status enqueue_batch_decode(ovf_model *m, ovf_session *const *ss, int n, cudaStream_t st) {
    const ovf_model_config &c = m->cfg;
    const int D = c.d_model, H = c.n_heads, KVH = c.n_kv_heads, hd = c.head_dim, QD = H * hd, KD = KVH * hd;
    const RowBufs rb{ActRows{m->baq, m->bas, m->bab}, m->bx, m->ba, m->bn, m->bq, m->bk, m->bv, m->batt,
                     m->bg, m->bu, m->bh};
    ovf_status r;
    if ((r = launch_embed_rows(m->btok, n, m->embed.type, m->embed.data, m->embed.scales, D, m->bx, st))) return r;
    for (int l = 0; l < c.n_layers; ++l) {
        const DevLayer &L = m->layers[l];
        if ((r = rows_norm_qkv(m, L, rb, n, st))) return r;
        for (int i = 0; i < n; ++i) {
            ovf_session *s = ss[i];
            const size_t esz = s->kv_dtype == OVF_KV_F32 ? 4 : s->kv_dtype == OVF_KV_Q8 ? 1 : 2;
            AttnParams a{};
            a.q = m->bq + (size_t)i * QD;
            a.k_new = m->bk + (size_t)i * KD;
            a.v_new = m->bv + (size_t)i * KD;
            a.kc = (__half *)((char *)s->kc + (size_t)l * KVH * s->max_ctx * hd * esz);
            a.vc = (__half *)((char *)s->vc + (size_t)l * KVH * s->max_ctx * hd * esz);
            if (s->kv_dtype == OVF_KV_Q8) {
                a.ks = s->ks + (size_t)l * KVH * s->max_ctx;
                a.vs = s->vs + (size_t)l * KVH * s->max_ctx;
            }
            a.out = m->batt + (size_t)i * QD;
            a.rope_cos = s->rope_cos;
            a.rope_sin = s->rope_sin;
            a.seq_len_host = s->pos + 1;
            a.partial = s->partial;
            a.counters = s->counters;
            a.split_half = c.rope_split_half;
            a.H = H;
            a.KVH = KVH;
            a.hd = hd;
            a.max_ctx = s->max_ctx;
            a.scale = 1.0f / sqrtf((float)hd);
            if ((r = launch_attention_exact(a, s->max_ctx, st, false, s->kv_dtype))) return r;
        }
        if ((r = rows_wo_ffn(m, L, rb, &m->bmoe, n, st))) return r;
    }
    // final norm, LM head rows, argmax per row
    if ((r = launch_rmsnorm_rows(m->bx, m->final_norm, m->bn, n, D, c.eps, nullptr, st))) return r;
    int fam = 0;
    if ((r = quantize_rows_for(rb.ar, m->lm_head, m->bn, n, D, &fam, st))) return r;
    if ((r = project_rows(rb.ar, m->lm_head, nullptr, m->blogits, n, st))) return r;
    if ((r = launch_argmax_rows(m->blogits, n, c.vocab, m->bargmax, st))) return r;
    for (int i = 0; i < n; ++i) {
        ovf_session *s = ss[i];
        OVF_CUDA_TRY(cudaMemcpyAsync(s->logits, m->blogits + (size_t)i * c.vocab, (size_t)c.vocab * 4,
                                     cudaMemcpyDeviceToDevice, st));
        if ((r = launch_batch_finish(s->step, s->pos, s->pos + 1, m->bargmax + i, s->tokens_log, st))) return r;
    }
    return OVF_OK;
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int d) {
        cudaGetDevice(&prev);
        cudaSetDevice(d);
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

}  // namespace

extern "C" {

// The exchange arena of a tensor-parallel rank: per layer the head outputs
// [n_heads][d_model] and the down terms [d_ff/256][d_model] of every rank,
// the logits [vocab], the ranks' argmax keys, the flags [2 * n_layers + 1]
// [world] and this rank's step epoch.
static ovf_status tp_arena_alloc(ovf_model *m) {
    const ovf_model_config &c = m->cfg;
    const DevLayer &L0 = m->layers[0];
    m->nb_down = c.n_experts ? 0 : L0.down.type == OVF_TYPE_Q8_0 ? c.d_ff / 32 : c.d_ff / 256;
    size_t o = 0;
    auto take = [&](size_t bytes) {
        const size_t at = o;
        o = (o + bytes + 255) & ~size_t(255);
        return at;
    };
    m->off_heads = take((size_t)c.n_layers * c.n_heads * c.d_model * 4);
    m->off_terms = c.n_experts ? 0 : take((size_t)c.n_layers * m->nb_down * c.d_model * 4);
    m->off_moe = c.n_experts ? take((size_t)c.n_layers * c.n_experts_used * c.d_model * 4) : 0;
    m->off_logits = take((size_t)c.vocab * 4);
    m->off_keys = take((size_t)m->tp_world * 8);
    m->off_flags = take((size_t)(2 * c.n_layers + 1) * m->tp_world * 4);
    m->off_epoch = take(16);
    m->arena_bytes = o;
    ovf_status st = dalloc(m->allocs, (void **)&m->arena, o);
    if (!st) st = cuda_status(cudaMemset(m->arena, 0, o), "arena memset");
    return st;
}

static ovf_status model_create(int32_t device, const ovf_model_config *cfg, const ovf_tensor *t, int32_t n_tensors,
                               int32_t rank, int32_t world, ovf_model **out) {
    OVF_CHECK_ARG(cfg && t && out, "ovf_model_create: null argument");
    const ovf_model_config &c = *cfg;
    OVF_CHECK_ARG(c.n_layers > 0 && c.d_model > 0 && c.n_heads > 0 && c.n_kv_heads > 0 && c.head_dim > 0 &&
                      c.d_ff > 0 && c.vocab > 0,
                  "ovf_model_create: config dimensions must be positive");
    OVF_CHECK_ARG(c.n_heads % c.n_kv_heads == 0, "ovf_model_create: n_heads must be a multiple of n_kv_heads");
    OVF_CHECK_ARG(c.head_dim % 32 == 0 && c.head_dim <= 256, "ovf_model_create: head_dim must be a multiple of 32, <= 256");
    OVF_CHECK_ARG(c.n_experts >= 0 && c.n_experts <= 64, "ovf_model_create: n_experts must be in [0, 64]");
    OVF_CHECK_ARG(c.n_experts == 0 || (c.n_experts_used >= 1 && c.n_experts_used <= 8 &&
                                       c.n_experts_used <= c.n_experts),
                  "ovf_model_create: n_experts_used must be in [1, min(8, n_experts)]");
    OVF_CHECK_ARG(n_tensors == c.n_layers * OVF_TENSORS_PER_LAYER + 3, "ovf_model_create: expected %d tensors, got %d",
                  c.n_layers * OVF_TENSORS_PER_LAYER + 3, n_tensors);
    int ndev = 0;
    OVF_CUDA_TRY(cudaGetDeviceCount(&ndev));
    OVF_CHECK_ARG(device >= 0 && device < ndev, "ovf_model_create: device %d not present", device);
    OVF_CHECK_ARG(world >= 1 && world <= 8 && rank >= 0 && rank < world, "ovf_model_create: bad rank %d of %d", rank,
                  world);
    const bool tp = world > 1;
    if (tp) {
        OVF_CHECK_ARG(c.n_experts == 0 || c.n_experts % world == 0,
                      "expert parallelism: %d experts do not split over %d ranks", c.n_experts, world);
        OVF_CHECK_ARG(c.n_kv_heads % world == 0, "tensor parallelism: %d KV heads do not split over %d ranks",
                      c.n_kv_heads, world);
        OVF_CHECK_ARG(c.n_experts > 0 || (c.d_ff % world == 0 && (c.d_ff / world) % 256 == 0),
                      "tensor parallelism: d_ff %d must split into multiples of 256", c.d_ff);
        OVF_CHECK_ARG(c.vocab % world == 0, "tensor parallelism: vocab %d must split evenly", c.vocab);
    }
    DeviceGuard guard(device);
    ovf_model *m = new ovf_model();
    m->device = device;
    m->cfg = c;
    m->tp_rank = rank;
    m->tp_world = world;
    m->h_loc = c.n_heads / world;
    m->kvh_loc = c.n_kv_heads / world;
    m->ff_loc = c.n_experts ? c.d_ff : c.d_ff / world;  // experts stay whole (expert parallel)
    m->v_loc = c.vocab / world;
    m->layers.resize(c.n_layers);
    const int64_t D = c.d_model, hd = c.head_dim, QD = (int64_t)c.n_heads * hd, KD = (int64_t)c.n_kv_heads * hd;
    const int64_t QDl = (int64_t)m->h_loc * hd, KDl = (int64_t)m->kvh_loc * hd, FFl = m->ff_loc;
    const int64_t q0 = (int64_t)rank * QDl, k0 = (int64_t)rank * KDl, f0 = (int64_t)rank * FFl;
    ovf_status st = OVF_OK;
    std::vector<uint8_t> colbuf;
    for (int l = 0; l < c.n_layers && !st; ++l) {
        const ovf_tensor *lt = t + (size_t)l * OVF_TENSORS_PER_LAYER;
        DevLayer &L = m->layers[l];
        if (!st) st = upload_vec(m, lt[0], D, &L.attn_norm, "attn_norm");
        if (!tp) {
            if (!st) st = upload_matrix(m, lt[1], QD, D, false, &L.wq, "attn_q");
            if (!st) st = upload_matrix(m, lt[2], KD, D, false, &L.wk, "attn_k");
            if (!st) st = upload_matrix(m, lt[3], KD, D, false, &L.wv, "attn_v");
            if (!st) st = upload_matrix(m, lt[4], D, QD, true, &L.wo, "attn_output");
            if (!st) st = upload_vec(m, lt[5], QD, &L.bq, "attn_q.bias");
            if (!st) st = upload_vec(m, lt[6], KD, &L.bk, "attn_k.bias");
            if (!st) st = upload_vec(m, lt[7], KD, &L.bv, "attn_v.bias");
        } else {
            // this rank's heads: Q/K/V rows, Wo columns (shard-aware upload)
            for (int i = 1; i <= 4 && !st; ++i)
                if (!lt[i].data) {
                    set_error("layer %d: attention weights are required", l);
                    st = OVF_EINVAL;
                }
            if (!st) OVF_CHECK_ARG(lt[1].rows == QD && lt[2].rows == KD && lt[3].rows == KD && lt[4].cols == QD,
                                   "layer %d: attention shapes", l);
            if (!st) st = upload_matrix(m, host_rows(lt[1], q0, QDl), QDl, D, false, &L.wq, "attn_q");
            if (!st) st = upload_matrix(m, host_rows(lt[2], k0, KDl), KDl, D, false, &L.wk, "attn_k");
            if (!st) st = upload_matrix(m, host_rows(lt[3], k0, KDl), KDl, D, false, &L.wv, "attn_v");
            if (!st) st = upload_wo_local(m, lt[4], D, QD, q0, QDl, &L.wo);
            if (!st) st = upload_vec(m, host_vec_slice(lt[5], q0, QDl), QDl, &L.bq, "attn_q.bias");
            if (!st) st = upload_vec(m, host_vec_slice(lt[6], k0, KDl), KDl, &L.bk, "attn_k.bias");
            if (!st) st = upload_vec(m, host_vec_slice(lt[7], k0, KDl), KDl, &L.bv, "attn_v.bias");
        }
        if (!st) st = upload_vec(m, lt[8], D, &L.bo, "attn_output.bias");
        if (!st) st = upload_vec(m, lt[9], D, &L.ffn_norm, "ffn_norm");
        const int64_t E = c.n_experts > 0 ? c.n_experts : 1;
        if (tp && c.n_experts > 0) {
            // expert parallel: this rank's experts e (e % world == rank), stacked
            // in order as local experts e / world
            const int64_t El = c.n_experts / world;
            for (int i = 10; i <= 12 && !st; ++i)
                if (!lt[i].data || lt[i].rows != E * (i == 12 ? D : c.d_ff)) {
                    set_error("layer %d: expert weights must hold n_experts matrices", l);
                    st = OVF_EINVAL;
                }
            std::vector<uint8_t> gb, ub, db;
            auto gather = [&](const ovf_tensor &t, int64_t rows_e, std::vector<uint8_t> &buf) {
                const int64_t eb = rows_e * host_row_bytes(t.type, t.cols);
                buf.resize((size_t)(El * eb));
                for (int64_t j = 0; j < El; ++j)
                    memcpy(buf.data() + j * eb, static_cast<const char *>(t.data) + (j * world + rank) * eb, (size_t)eb);
                return ovf_tensor{t.type, buf.data(), El * rows_e, t.cols};
            };
            if (!st) st = upload_matrix(m, gather(lt[10], c.d_ff, gb), El * c.d_ff, D, false, &L.gate, "ffn_gate");
            if (!st) st = upload_matrix(m, gather(lt[11], c.d_ff, ub), El * c.d_ff, D, false, &L.up, "ffn_up");
            if (!st) st = upload_matrix(m, gather(lt[12], D, db), El * D, c.d_ff, false, &L.down, "ffn_down");
        } else if (!tp) {
            if (!st) st = upload_matrix(m, lt[10], E * c.d_ff, D, false, &L.gate, "ffn_gate");
            if (!st) st = upload_matrix(m, lt[11], E * c.d_ff, D, false, &L.up, "ffn_up");
            if (!st) st = upload_matrix(m, lt[12], E * D, c.d_ff, false, &L.down, "ffn_down");
        } else {
            // this rank's FFN slice: gate/up rows, down columns
            if (!st && (!lt[10].data || !lt[11].data || !lt[12].data || lt[12].cols != c.d_ff || lt[12].rows != D)) {
                set_error("layer %d: FFN weights are required", l);
                st = OVF_EINVAL;
            }
            if (!st) st = upload_matrix(m, host_rows(lt[10], f0, FFl), FFl, D, false, &L.gate, "ffn_gate");
            if (!st) st = upload_matrix(m, host_rows(lt[11], f0, FFl), FFl, D, false, &L.up, "ffn_up");
            if (!st) st = upload_matrix(m, host_cols(lt[12], f0, FFl, colbuf), D, FFl, false, &L.down, "ffn_down");
        }
        if (!st && c.n_experts > 0) {
            // Mixtral: ffn_gate_inp as the input-major F32 router; experts stacked
            ovf_tensor rt = lt[13];
            if (!rt.data || rt.type != OVF_TYPE_F32 || rt.rows != D || rt.cols != c.n_experts) {
                set_error("layer %d: MoE router must be F32 [d_model x n_experts] (input-major)", l);
                st = OVF_EINVAL;
            } else {
                ovf_tensor flat{OVF_TYPE_F32, rt.data, 1, D * c.n_experts};
                st = upload_vec(m, flat, D * c.n_experts, &L.router, "ffn_gate_inp");
            }
            if (!st && (L.gate.type != L.up.type)) {
                set_error("layer %d: MoE gate and up experts must share a type", l);
                st = OVF_EINVAL;
            }
            if (!st) {
                expert_strides(L.gate, c.d_ff, &L.gu_wstride, &L.gu_sstride);
                expert_strides(L.down, D, &L.d_wstride, &L.d_sstride);
                if (L.gu_wstride % 16 || L.gu_sstride % 16 || L.d_wstride % 16 || L.d_sstride % 16) {
                    set_error("layer %d: expert matrices must be multiples of 16 bytes", l);
                    st = OVF_EINVAL;
                }
                // a decode step streams n_experts_used of the n_experts (over all ranks)
                const int64_t per = 2 * (L.gu_wstride + L.gu_sstride) + L.d_wstride + L.d_sstride;
                m->weight_bytes -= (int64_t)(c.n_experts / world) * per;
                m->weight_bytes += (int64_t)c.n_experts_used * per / world;
            }
        }
        if (!st && (!L.attn_norm || !L.ffn_norm)) {
            set_error("layer %d: norms are required", l);
            st = OVF_EINVAL;
        }
    }
    const ovf_tensor *tail = t + (size_t)c.n_layers * OVF_TENSORS_PER_LAYER;
    if (!st) {
        // Embedding (GgufLlamaLoader.cs:546-572): K-quants stay; Q8_0 is held
        // de-interleaved (its row decode equals the reference's F32 dequant);
        // F32 stays F32.
        const ovf_tensor &e = tail[0];
        if (!e.data || e.rows != c.vocab || e.cols != D) {
            set_error("token_embd must be vocab x d_model");
            st = OVF_EINVAL;
        } else if (e.type == OVF_TYPE_F32) {
            m->embed.type = OVF_TYPE_F32;
            m->embed.rows = e.rows;
            m->embed.cols = e.cols;
            st = dalloc(m->allocs, (void **)&m->embed.data, D * c.vocab * 4);
            if (!st) st = cuda_status(cudaMemcpy(m->embed.data, e.data, D * c.vocab * 4, cudaMemcpyHostToDevice), "embed");
        } else {
            st = upload_matrix(m, e, c.vocab, D, false, &m->embed, "token_embd");
            m->weight_bytes -= (m->embed.type == OVF_TYPE_Q8_0) ? (int64_t)c.vocab * D * 9 / 8
                                                                : tensor_bytes(m->embed.type, c.vocab, D);
        }
    }
    if (!st) st = upload_vec(m, tail[1], D, &m->final_norm, "output_norm");
    if (!st && tp) {
        // this rank's vocabulary rows of the LM head (tied: of the embedding)
        const ovf_tensor &o = tail[2];
        const int64_t v0 = (int64_t)rank * m->v_loc, vl = m->v_loc;
        if (o.data && o.type >= 0) {
            st = upload_matrix(m, host_rows(o, v0, vl), vl, D, o.type == OVF_TYPE_F32, &m->lm_head, "output");
        } else if (m->embed.type == OVF_TYPE_F32) {
            ovf_tensor tt{OVF_TYPE_F32, tail[0].data, c.vocab, D};
            st = upload_matrix(m, host_rows(tt, v0, vl), vl, D, true, &m->lm_head, "output(tied)");
        } else {
            m->lm_head = m->embed;
            m->lm_head.owns = false;
            m->lm_head.rows = vl;
            if (m->embed.type == OVF_TYPE_Q8_0) {
                m->lm_head.data = m->embed.data + v0 * D;
                m->lm_head.scales = m->embed.scales + v0 * D / 32;
                m->weight_bytes += vl * D * 9 / 8;
            } else {
                m->lm_head.data = m->embed.data + v0 * host_row_bytes(m->embed.type, D);
                m->weight_bytes += tensor_bytes(m->embed.type, vl, D);
            }
        }
    }
    if (!st && !tp) {
        const ovf_tensor &o = tail[2];
        if (o.data && o.type >= 0) {
            st = upload_matrix(m, o, c.vocab, D, o.type == OVF_TYPE_F32, &m->lm_head, "output");
        } else if (m->embed.type == OVF_TYPE_F32) {
            // Tied F32 embedding: the reference re-quantizes it to Q8_0 (GgufLlamaLoader.cs:478-483).
            ovf_tensor tt{OVF_TYPE_F32, tail[0].data, c.vocab, D};
            st = upload_matrix(m, tt, c.vocab, D, true, &m->lm_head, "output(tied)");
        } else {
            m->lm_head = m->embed;  // tied: same resident bytes
            m->lm_head.owns = false;
            m->weight_bytes += (m->embed.type == OVF_TYPE_Q8_0) ? (int64_t)c.vocab * D * 9 / 8
                                                                : tensor_bytes(m->embed.type, c.vocab, D);
        }
    }
    if (!st && tp) st = tp_arena_alloc(m);
    if (st) {
        ovf_model_destroy(m);
        return st;
    }
    *out = m;
    return OVF_OK;
}

ovf_status ovf_model_create(int32_t device, const ovf_model_config *cfg, const ovf_tensor *t, int32_t n_tensors,
                            ovf_model **out) {
    return model_create(device, cfg, t, n_tensors, 0, 1, out);
}

ovf_status ovf_model_create_tp(int32_t device, const ovf_model_config *cfg, const ovf_tensor *t, int32_t n_tensors,
                               int32_t rank, int32_t world, ovf_model **out) {
    return model_create(device, cfg, t, n_tensors, rank, world, out);
}

ovf_status ovf_model_tp_export(ovf_model *m, void *handle_out) {
    OVF_CHECK_ARG(m && handle_out, "tp_export: null argument");
    OVF_CHECK_ARG(m->tp_world > 1 && m->arena, "tp_export: not a tensor-parallel model");
    DeviceGuard guard(m->device);
    cudaIpcMemHandle_t h;
    OVF_CUDA_TRY(cudaIpcGetMemHandle(&h, m->arena));
    memcpy(handle_out, &h, sizeof(h));
    return OVF_OK;
}

ovf_status ovf_model_tp_connect(ovf_model *m, const void *handles) {
    OVF_CHECK_ARG(m && handles, "tp_connect: null argument");
    OVF_CHECK_ARG(m->tp_world > 1 && m->arena, "tp_connect: not a tensor-parallel model");
    OVF_CHECK_ARG(!m->tp_ready, "tp_connect: already connected");
    DeviceGuard guard(m->device);
    for (int w = 0; w < m->tp_world; ++w) {
        if (w == m->tp_rank) {
            m->peer[w] = m->arena;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const char *>(handles) + (size_t)w * sizeof(h), sizeof(h));
        void *p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int v = 0; v < w; ++v)
                if (v != m->tp_rank && m->peer[v]) cudaIpcCloseMemHandle(m->peer[v]);
            return cuda_status(e, "cudaIpcOpenMemHandle");
        }
        m->peer[w] = static_cast<char *>(p);
    }
    m->tp_ready = true;
    return OVF_OK;
}

ovf_status ovf_model_destroy(ovf_model *m) {
    if (!m) return OVF_OK;
    DeviceGuard guard(m->device);
    if (m->btok_host) cudaFreeHost(m->btok_host);
    if (m->bmoe.host) cudaFreeHost(m->bmoe.host);
    if (m->tp_ready)
        for (int w = 0; w < m->tp_world; ++w)
            if (w != m->tp_rank && m->peer[w]) cudaIpcCloseMemHandle(m->peer[w]);
    for (void *p : m->allocs) cudaFree(p);
    delete m;
    return OVF_OK;
}

int64_t ovf_model_weight_bytes(const ovf_model *m) { return m ? m->weight_bytes : 0; }

ovf_status ovf_session_create(ovf_model *m, int32_t max_ctx, ovf_session **out) {
    return ovf_session_create_kv(m, max_ctx, OVF_KV_F32, out);
}

ovf_status ovf_session_create_kv(ovf_model *m, int32_t max_ctx, int32_t kv_dtype, ovf_session **out) {
    OVF_CHECK_ARG(m && out, "ovf_session_create: null argument");
    OVF_CHECK_ARG(max_ctx > 0 && max_ctx <= (1 << 20), "ovf_session_create: bad max_ctx");
    OVF_CHECK_ARG(kv_dtype == OVF_KV_F32 || kv_dtype == OVF_KV_Q8 || kv_dtype == OVF_KV_F16,
                  "ovf_session_create: unknown KV dtype %d", kv_dtype);
    OVF_CHECK_ARG(attn_exact_supported(m->cfg.head_dim), "ovf_session_create: head_dim %d unsupported",
                  m->cfg.head_dim);
    OVF_CHECK_ARG(max_ctx <= attn_exact_max_seq(m->cfg.head_dim), "ovf_session_create: max_ctx too large");
    DeviceGuard guard(m->device);
    ovf_session *s = new ovf_session();
    s->m = m;
    s->max_ctx = max_ctx;
    s->kv_dtype = kv_dtype;
    const ovf_model_config &c = m->cfg;
    // tensor parallel: this rank's heads and FFN rows only
    const size_t D = c.d_model, QD = (size_t)m->h_loc * c.head_dim, KD = (size_t)m->kvh_loc * c.head_dim;
    const size_t FF = (size_t)m->ff_loc;
    const size_t kv = (size_t)c.n_layers * KD * max_ctx;
    ovf_status st = OVF_OK;
    auto A = [&](void **p, size_t bytes) {
        if (!st) st = dalloc(s->allocs, p, bytes);
    };
    const size_t esz = kv_dtype == OVF_KV_F32 ? 4 : kv_dtype == OVF_KV_Q8 ? 1 : 2;
    A((void **)&s->kc, kv * esz);
    A((void **)&s->vc, kv * esz);
    if (kv_dtype == OVF_KV_Q8) {
        A((void **)&s->ks, kv / c.head_dim * 4);
        A((void **)&s->vs, kv / c.head_dim * 4);
    }
    A((void **)&s->hidden, D * 4);
    A((void **)&s->after, D * 4);
    A((void **)&s->q, QD * 4);
    A((void **)&s->k, KD * 4);
    A((void **)&s->v, KD * 4);
    A((void **)&s->attn, QD * 4);
    A((void **)&s->h, FF * 4);
    A((void **)&s->gtmp, FF * 4);
    A((void **)&s->utmp, FF * 4);
    A((void **)&s->logits, (size_t)c.vocab * 4);
    A((void **)&s->rope_cos, (size_t)max_ctx * c.head_dim / 2 * 4);
    A((void **)&s->rope_sin, (size_t)max_ctx * c.head_dim / 2 * 4);
    A((void **)&s->partial, (size_t)attn_scratch_bytes(m->h_loc, m->kvh_loc, c.head_dim));
    A((void **)&s->counters, (size_t)m->kvh_loc * 4);
    A((void **)&s->norm_s, 2 * 4);
    if (env_flag("OVF_TRACE")) {
        s->trace_cap = 8 * c.n_layers + 16;
        A((void **)&s->trace, (size_t)s->trace_cap * sizeof(TraceSlot));
    }
    A((void **)&s->tokens_log, (size_t)(max_ctx + 1) * 4);
    A((void **)&s->step, sizeof(DevStep));
    A((void **)&s->err_slot, sizeof(int));
    if (c.n_experts > 0) {
        A((void **)&s->msel, (size_t)c.n_experts_used * 4);
        A((void **)&s->mw, (size_t)c.n_experts_used * 4);
        A((void **)&s->mh, (size_t)c.n_experts_used * c.d_ff * 4);
        A((void **)&s->meo, (size_t)c.n_experts_used * D * 4);
    }
    if (!st) st = cuda_status(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking), "stream");
    if (!st) st = cuda_status(cudaMemset(s->counters, 0, (size_t)m->kvh_loc * 4), "memset");
    s->prefill_single = m->tp_world > 1;  // the batched prefill is not split over ranks
    if (!st) st = cuda_status(cudaMemset(s->step, 0, sizeof(DevStep)), "memset");
    if (!st) st = cuda_status(cudaMemset(s->kc, 0, kv * esz), "memset");
    if (!st) st = cuda_status(cudaMemset(s->vc, 0, kv * esz), "memset");
    if (!st) st = fill_rope_tables(s);
    if (!st) {
        s->pinned_cap = max_ctx + 1;
        st = cuda_status(cudaMallocHost(&s->pinned_tok, (size_t)s->pinned_cap * 4), "cudaMallocHost");
    }
    if (st) {
        ovf_session_destroy(s);
        return st;
    }
    *out = s;
    return OVF_OK;
}

ovf_status ovf_session_destroy(ovf_session *s) {
    if (!s) return OVF_OK;
    DeviceGuard guard(s->m->device);
    if (s->stream) cudaStreamSynchronize(s->stream);
    prof_report();
    trace_report(s);
    if (s->graph_logits) cudaGraphExecDestroy(s->graph_logits);
    if (s->graph_nologits) cudaGraphExecDestroy(s->graph_nologits);
    for (void *p : s->allocs) cudaFree(p);
    if (s->pinned_tok) cudaFreeHost(s->pinned_tok);
    if (s->pmoe.host) cudaFreeHost(s->pmoe.host);
    if (s->stream) cudaStreamDestroy(s->stream);
    delete s;
    return OVF_OK;
}

ovf_status ovf_session_reset(ovf_session *s) {
    OVF_CHECK_ARG(s, "ovf_session_reset: null session");
    DeviceGuard guard(s->m->device);
    OVF_CUDA_TRY(cudaMemsetAsync(s->step, 0, sizeof(DevStep), s->stream));
    OVF_CUDA_TRY(cudaStreamSynchronize(s->stream));
    s->pos = 0;
    s->n_logits = 0;
    s->needs_reset = false;
    return OVF_OK;
}

int32_t ovf_session_position(const ovf_session *s) { return s ? s->pos : -1; }

// Ends a synchronous call: moves the device error word into `slot` (read and
// cleared in one atomic step, after the call's kernels), waits for the stream
// and reports a bounded wait that gave up as OVF_ETIMEDOUT.
static ovf_status finish_call(cudaStream_t st, int *slot) {
    ovf_status r = launch_take_error(slot, st);
    if (r) return r;
    int code = 0;
    OVF_CUDA_TRY(cudaMemcpyAsync(&code, slot, sizeof(int), cudaMemcpyDeviceToHost, st));
    OVF_CUDA_TRY(cudaStreamSynchronize(st));
    if (code) {
        set_error("device wait timed out (code %d)", code);
        return OVF_ETIMEDOUT;
    }
    return OVF_OK;
}

static ovf_status decode_impl(ovf_session *s, const int32_t *tokens, int32_t n, float *logits_host, int32_t *argmax_out) {
    OVF_CHECK_ARG(s, "decode: null session");
    if (s->needs_reset) {
        set_error("session state is undefined after a failed batch call; call ovf_session_reset");
        return OVF_ESTATE;
    }
    OVF_CHECK_ARG(n >= 0 && (n == 0 || tokens), "decode: bad token array");
    if (s->m->tp_world > 1 && !s->m->tp_ready) {
        set_error("tensor-parallel model: call ovf_model_tp_connect on every rank first");
        return OVF_ESTATE;
    }
    OVF_CHECK_ARG(s->pos + n <= s->max_ctx, "KV cache is full (ContextLength=%d, position %d, %d new tokens)", s->max_ctx,
                  s->pos, n);
    if (n == 0) return OVF_OK;
    for (int i = 0; i < n; ++i)
        OVF_CHECK_ARG(tokens[i] >= 0 && tokens[i] < s->m->cfg.vocab, "token id %d out of range", tokens[i]);
    DeviceGuard guard(s->m->device);
    OVF_CUDA_TRY(cudaStreamSynchronize(s->stream));
    int done = 0;
    if (n >= kPrefillThreshold && !s->prefill_single) {
        // the batched path (n <= max_ctx <= pinned_cap)
        ovf_status r = prefill_alloc(s);
        if (r) return r;
        memcpy(s->pinned_tok, tokens, (size_t)n * 4);
        OVF_CUDA_TRY(cudaMemcpyAsync(s->ptok, s->pinned_tok, (size_t)n * 4, cudaMemcpyHostToDevice, s->stream));
        if ((r = enqueue_prefill_batched(s, n))) return r;
        s->pos += n;
        s->n_logits += 1;
        done = n;
    }
    while (done < n) {
        const int chunk = std::min(n - done, s->pinned_cap);
        memcpy(s->pinned_tok, tokens + done, (size_t)chunk * 4);
        for (int i = 0; i < chunk; ++i) {
            const bool last = done + i == n - 1;
            OVF_CUDA_TRY(cudaMemcpyAsync(&s->step->token, s->pinned_tok + i, 4, cudaMemcpyHostToDevice, s->stream));
            ovf_status r = run_step(s, last);
            if (r) return r;
        }
        OVF_CUDA_TRY(cudaStreamSynchronize(s->stream));
        done += chunk;
    }
    if (logits_host)
        OVF_CUDA_TRY(cudaMemcpyAsync(logits_host, s->logits, (size_t)s->m->cfg.vocab * 4, cudaMemcpyDeviceToHost, s->stream));
    if (argmax_out) OVF_CUDA_TRY(cudaMemcpyAsync(argmax_out, &s->step->token, 4, cudaMemcpyDeviceToHost, s->stream));
    return finish_call(s->stream, s->err_slot);
}

ovf_status ovf_session_decode(ovf_session *s, int32_t token, float *logits_host, int32_t *argmax_out) {
    return decode_impl(s, &token, 1, logits_host, argmax_out);
}

ovf_status ovf_session_prefill(ovf_session *s, const int32_t *tokens, int32_t n, float *logits_host,
                               int32_t *argmax_out) {
    return decode_impl(s, tokens, n, logits_host, argmax_out);
}

ovf_status ovf_session_generate_greedy(ovf_session *s, int32_t n_steps, int32_t *tokens_out) {
    OVF_CHECK_ARG(s && n_steps >= 0 && (n_steps == 0 || tokens_out), "generate: bad arguments");
    OVF_CHECK_ARG(s->n_logits > 0, "Session is empty. Call Reset with at least one prompt token first.");
    if (s->m->tp_world > 1 && !s->m->tp_ready) {
        set_error("tensor-parallel model: call ovf_model_tp_connect on every rank first");
        return OVF_ESTATE;
    }
    OVF_CHECK_ARG(s->pos + n_steps <= s->max_ctx, "KV cache is full (ContextLength=%d)", s->max_ctx);
    DeviceGuard guard(s->m->device);
    const int first = s->n_logits - 1;  // the token sampled from the current logits
    for (int i = 0; i < n_steps; ++i) {
        ovf_status r = run_step(s, true);
        if (r) return r;
    }
    OVF_CUDA_TRY(cudaMemcpyAsync(tokens_out, s->tokens_log + first, (size_t)n_steps * 4, cudaMemcpyDeviceToHost, s->stream));
    return finish_call(s->stream, s->err_slot);
}

void *ovf_session_stream(const ovf_session *s) { return s ? (void *)s->stream : nullptr; }

ovf_status ovf_session_decode_batch(ovf_session *const *sessions, int32_t n, const int32_t *tokens,
                                    float *logits_host, int32_t *argmax_out) {
    OVF_CHECK_ARG(sessions && tokens && n > 0, "decode batch: bad arguments");
    OVF_CHECK_ARG(n <= kBatchMax, "decode batch: at most %d sessions per call, got %d", kBatchMax, n);
    ovf_model *m = sessions[0] ? sessions[0]->m : nullptr;
    OVF_CHECK_ARG(m, "decode batch: null session");
    if (m->tp_world > 1) {
        set_error("decode batch: not available on a tensor-parallel model");
        return OVF_EUNSUPPORTED;
    }
    for (int i = 0; i < n; ++i) {
        ovf_session *s = sessions[i];
        OVF_CHECK_ARG(s && s->m == m, "decode batch: session %d is null or of another model", i);
        for (int j = 0; j < i; ++j) OVF_CHECK_ARG(sessions[j] != s, "decode batch: session %d repeated", i);
        OVF_CHECK_ARG(s->pos + 1 <= s->max_ctx, "KV cache is full (ContextLength=%d) in session %d", s->max_ctx, i);
        OVF_CHECK_ARG(tokens[i] >= 0 && tokens[i] < m->cfg.vocab, "token id %d out of range", tokens[i]);
    }
    for (int i = 0; i < n; ++i)
        if (sessions[i]->needs_reset) {
            set_error("decode batch: session %d needs ovf_session_reset after a failed batch call", i);
            return OVF_ESTATE;
        }
    bool idle = false;
    if (!m->batch_busy.compare_exchange_strong(idle, true)) {
        set_error("decode batch: another batch call on this model is in flight");
        return OVF_EBUSY;
    }
    struct BusyRelease {
        std::atomic<bool> &f;
        ~BusyRelease() { f.store(false); }
    } busy_release{m->batch_busy};
    DeviceGuard guard(m->device);
    ovf_status r = batch_alloc(m);
    if (r) return r;
    for (int i = 0; i < n; ++i) OVF_CUDA_TRY(cudaStreamSynchronize(sessions[i]->stream));
    const cudaStream_t st = sessions[0]->stream;
    memcpy(m->btok_host, tokens, (size_t)n * 4);
    OVF_CUDA_TRY(cudaMemcpyAsync(m->btok, m->btok_host, (size_t)n * 4, cudaMemcpyHostToDevice, st));
    if ((r = enqueue_batch_decode(m, sessions, n, st))) {
        // some sessions may already have appended K/V rows or advanced their
        // device step: their state no longer matches `pos`
        for (int i = 0; i < n; ++i) sessions[i]->needs_reset = true;
        return r;
    }
    for (int i = 0; i < n; ++i) {
        sessions[i]->pos += 1;
        sessions[i]->n_logits += 1;
    }
    if (logits_host)
        OVF_CUDA_TRY(cudaMemcpyAsync(logits_host, m->blogits, (size_t)n * m->cfg.vocab * 4, cudaMemcpyDeviceToHost, st));
    if (argmax_out) OVF_CUDA_TRY(cudaMemcpyAsync(argmax_out, m->bargmax, (size_t)n * 4, cudaMemcpyDeviceToHost, st));
    return finish_call(st, sessions[0]->err_slot);
}

ovf_status ovf_session_set_option(ovf_session *s, int32_t option, int32_t value) {
    OVF_CHECK_ARG(s, "set_option: null session");
    switch (option) {
        case OVF_OPT_PREFILL_SINGLE: s->prefill_single = value != 0; return OVF_OK;
        default: OVF_CHECK_ARG(false, "set_option: unknown option %d", option);
    }
}

// ------------------------------------------------ speculative verify / KV
// CachedLlamaSession.GenerateSpeculativeCore's verify forward (:468-477):
// the rows [t0, drafts...] through the batched stack at positions pos..,
// every row to logits.  Each row's arithmetic is a decode step's, so row j's
// logits equal those a single-token decode of tokens[0..j] would give.
constexpr int kVerifyMax = 64;

ovf_status ovf_session_verify(ovf_session *s, const int32_t *tokens, int32_t n, float *logits_host,
                              int32_t *argmax_out) {
    OVF_CHECK_ARG(s && tokens && n >= 1, "verify: bad arguments");
    OVF_CHECK_ARG(n <= kVerifyMax, "verify: at most %d rows per call, got %d", kVerifyMax, n);
    if (s->m->tp_world > 1) {
        set_error("verify: not available on a tensor-parallel model");
        return OVF_EUNSUPPORTED;
    }
    if (s->needs_reset) {
        set_error("session state is undefined after a failed batch call; call ovf_session_reset");
        return OVF_ESTATE;
    }
    OVF_CHECK_ARG(s->pos + n <= s->max_ctx, "KV cache is full (ContextLength=%d, position %d, %d new tokens)",
                  s->max_ctx, s->pos, n);
    for (int i = 0; i < n; ++i)
        OVF_CHECK_ARG(tokens[i] >= 0 && tokens[i] < s->m->cfg.vocab, "token id %d out of range", tokens[i]);
    DeviceGuard guard(s->m->device);
    OVF_CUDA_TRY(cudaStreamSynchronize(s->stream));
    ovf_status r = prefill_alloc(s);
    if (r) return r;
    if (!s->vlogits) {
        if ((r = dalloc(s->allocs, (void **)&s->vlogits, (size_t)kVerifyMax * s->m->cfg.vocab * 4))) return r;
        if ((r = dalloc(s->allocs, (void **)&s->vargmax, (size_t)kVerifyMax * 4))) return r;
    }
    memcpy(s->pinned_tok, tokens, (size_t)n * 4);
    OVF_CUDA_TRY(cudaMemcpyAsync(s->ptok, s->pinned_tok, (size_t)n * 4, cudaMemcpyHostToDevice, s->stream));
    if ((r = enqueue_prefill_batched(s, n, true))) {
        s->needs_reset = true;
        return r;
    }
    s->pos += n;
    s->n_logits += 1;
    if (logits_host)
        OVF_CUDA_TRY(cudaMemcpyAsync(logits_host, s->vlogits, (size_t)n * s->m->cfg.vocab * 4, cudaMemcpyDeviceToHost,
                                     s->stream));
    if (argmax_out) OVF_CUDA_TRY(cudaMemcpyAsync(argmax_out, s->vargmax, (size_t)n * 4, cudaMemcpyDeviceToHost, s->stream));
    return finish_call(s->stream, s->err_slot);
}

// KeyValueCache.TruncateTo (Runtime/KeyValueCache.cs:246-258) as
// CachedLlamaSession.RollbackTo (:318) uses it: positions [length, pos) are
// dropped; their stale rows are overwritten before they are read again.
ovf_status ovf_session_truncate(ovf_session *s, int32_t length) {
    OVF_CHECK_ARG(s, "TruncateTo: null session");
    OVF_CHECK_ARG(length >= 0 && length <= s->pos, "TruncateTo %d must be in [0, CurrentLength=%d]", length, s->pos);
    DeviceGuard guard(s->m->device);
    ovf_status r = launch_set_step_pos(s->step, length > 0 ? length - 1 : 0, length, s->stream);
    if (r) return r;
    OVF_CUDA_TRY(cudaStreamSynchronize(s->stream));
    s->pos = length;
    return OVF_OK;
}

static size_t kv_elem_bytes(const ovf_session *s) {
    return s->kv_dtype == OVF_KV_F32 ? 4 : s->kv_dtype == OVF_KV_Q8 ? 1 : 2;
}

int64_t ovf_session_prefix_bytes(const ovf_session *s) {
    if (!s) return -1;
    const ovf_model_config &c = s->m->cfg;
    return (int64_t)c.n_layers * c.n_kv_heads * s->pos * c.head_dim * (int64_t)kv_elem_bytes(s);
}

// KeyValueCache.Snapshot (Runtime/KeyValueCache.cs:264-289) via
// CachedLlamaSession.SavePrefix (:231): the live rows [0, pos) of every
// (layer, KV head), packed [layer][kv_head][pos][head_dim] into the caller's
// host buffers (ovf_session_prefix_bytes each).  F32 (the reference's only
// snapshot type) and fp16 caches; a Q8 cache is rejected as the reference's
// ThrowIfQuantized does.
ovf_status ovf_session_save_prefix(const ovf_session *s, void *keys, void *values, int32_t *length_out) {
    OVF_CHECK_ARG(s && keys && values && length_out, "SavePrefix: null argument");
    if (s->kv_dtype == OVF_KV_Q8) {
        set_error("Snapshot is not supported for a quantized (Q8) KV cache");
        return OVF_EUNSUPPORTED;
    }
    DeviceGuard guard(s->m->device);
    const ovf_model_config &c = s->m->cfg;
    const size_t esz = kv_elem_bytes(s), run = (size_t)s->pos * c.head_dim * esz,
                 pitch = (size_t)s->max_ctx * c.head_dim * esz, lh = (size_t)c.n_layers * c.n_kv_heads;
    *length_out = s->pos;
    if (run == 0) return OVF_OK;
    OVF_CUDA_TRY(cudaMemcpy2DAsync(keys, run, s->kc, pitch, run, lh, cudaMemcpyDeviceToHost, s->stream));
    OVF_CUDA_TRY(cudaMemcpy2DAsync(values, run, s->vc, pitch, run, lh, cudaMemcpyDeviceToHost, s->stream));
    OVF_CUDA_TRY(cudaStreamSynchronize(s->stream));
    return OVF_OK;
}

// KeyValueCache.RestoreFrom (Runtime/KeyValueCache.cs:296-327) via
// CachedLlamaSession.RestorePrefix (:242): rows [0, length) of every
// (layer, KV head) from a packed prefix of the same model and cache type;
// the session's position becomes `length` (a copy, not a forward pass) and it
// holds no logits until the next prefill / decode.
ovf_status ovf_session_restore_prefix(ovf_session *s, const void *keys, const void *values, int32_t length) {
    OVF_CHECK_ARG(s && (length == 0 || (keys && values)), "RestorePrefix: null argument");
    if (s->kv_dtype == OVF_KV_Q8) {
        set_error("RestoreFrom is not supported for a quantized (Q8) KV cache");
        return OVF_EUNSUPPORTED;
    }
    OVF_CHECK_ARG(length >= 0 && length <= s->max_ctx, "Snapshot length %d exceeds cache MaxLength %d", length,
                  s->max_ctx);
    DeviceGuard guard(s->m->device);
    const ovf_model_config &c = s->m->cfg;
    const size_t esz = kv_elem_bytes(s), run = (size_t)length * c.head_dim * esz,
                 pitch = (size_t)s->max_ctx * c.head_dim * esz, lh = (size_t)c.n_layers * c.n_kv_heads;
    OVF_CUDA_TRY(cudaStreamSynchronize(s->stream));
    OVF_CUDA_TRY(cudaMemsetAsync(s->step, 0, sizeof(DevStep), s->stream));
    if (run) {
        OVF_CUDA_TRY(cudaMemcpy2DAsync(s->kc, pitch, keys, run, run, lh, cudaMemcpyHostToDevice, s->stream));
        OVF_CUDA_TRY(cudaMemcpy2DAsync(s->vc, pitch, values, run, run, lh, cudaMemcpyHostToDevice, s->stream));
    }
    ovf_status r = launch_set_step_pos(s->step, length > 0 ? length - 1 : 0, length, s->stream);
    if (r) return r;
    OVF_CUDA_TRY(cudaStreamSynchronize(s->stream));
    s->pos = length;
    s->n_logits = 0;
    s->needs_reset = false;
    return OVF_OK;
}

}  // extern "C"
