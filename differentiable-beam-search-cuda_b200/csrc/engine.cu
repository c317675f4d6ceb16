// Host orchestration of the device engine (see engine.h).
#include "engine.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

namespace dbs_host {

void check_cuda(cudaError_t err, const char* what) {
    if (err != cudaSuccess) {
        throw CudaFailure(std::string(what) + ": " + cudaGetErrorString(err));
    }
}

int pool_size(int beam_size, int multiplier) {
    const long long p = static_cast<long long>(beam_size) * static_cast<long long>(multiplier);
    if (p > 2147483647LL) throw std::overflow_error("relaxed pool size exceeds int range");
    return p > beam_size ? static_cast<int>(p) : beam_size;
}

int device_sm_count() {
    int dev = 0;
    check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    static std::mutex mu;
    static std::vector<int> cache;
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= static_cast<int>(cache.size())) cache.resize(dev + 1, 0);
    if (cache[dev] == 0) {
        int n = 0;
        check_cuda(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev), "sm count");
        cache[dev] = n;
    }
    return cache[dev];
}

// gnmt_length_penalty (src/differentiable_beam.cpp:277-282), evaluated on the
// host with the same float powf as the reference, plus its reciprocal
// 1.0f / pen as used by the scan and the backward.
static void penalty_tables(float alpha, int lmax, std::vector<float>& pen, std::vector<float>& inv) {
    pen.resize(lmax + 1);
    inv.resize(lmax + 1);
    for (int l = 0; l <= lmax; ++l) {
        float v = 1.0f;
        if (alpha != 0.0f) {
            const int ll = l < 1 ? 1 : l;
            v = std::pow((5.0f + static_cast<float>(ll)) / 6.0f, alpha);
        }
        pen[l] = v;
        volatile float one = 1.0f;
        inv[l] = one / v;
    }
}

Layout make_layout(const Options& opt, const std::vector<ExampleSpec>& ex, int V) {
    Layout L;
    const size_t B = ex.size();
    L.sel_offset.resize(B);
    L.pool_offset.resize(B);
    L.final_offset.resize(B);
    L.grad_offset.resize(B);
    L.sparse_offset.resize(B);
    L.P.resize(B);
    for (size_t b = 0; b < B; ++b) {
        const int P = pool_size(ex[b].K, opt.relaxed_pool_multiplier);
        L.P[b] = P;
        L.sel_offset[b] = L.sel_total;
        L.pool_offset[b] = L.pool_total;
        L.final_offset[b] = L.final_total;
        L.grad_offset[b] = L.grad_total;
        L.sparse_offset[b] = L.sparse_total;
        L.sel_total += static_cast<int64_t>(ex[b].T) * ex[b].K;
        L.pool_total += static_cast<int64_t>(ex[b].T) * P;
        L.final_total += ex[b].K;
        L.grad_total += static_cast<int64_t>(ex[b].T) * ex[b].K * V;
        L.sparse_total += static_cast<int64_t>(ex[b].T) * (ex[b].K + P);
    }
    return L;
}

namespace {

struct EventPair {
    cudaEvent_t a, b;
    int kernel;
};
std::mutex g_prof_mu;
bool g_prof_on = false;
std::vector<EventPair> g_prof_pending;
double g_prof_ms[kProfiledKernels] = {0};
long long g_prof_n[kProfiledKernels] = {0};

void prof_drain_locked() {
    for (EventPair& p : g_prof_pending) {
        float ms = 0.0f;
        if (cudaEventSynchronize(p.b) == cudaSuccess && cudaEventElapsedTime(&ms, p.a, p.b) == cudaSuccess) {
            g_prof_ms[p.kernel] += ms;
            g_prof_n[p.kernel] += 1;
        } else {
            cudaGetLastError();
        }
        cudaEventDestroy(p.a);
        cudaEventDestroy(p.b);
    }
    g_prof_pending.clear();
}

// Records an event pair around one launch on `stream` when profiling is on.
struct ProfileScope {
    cudaEvent_t a = nullptr, b = nullptr;
    cudaStream_t s;
    int kernel;
    ProfileScope(int k, cudaStream_t stream) : s(stream), kernel(k) {
        bool on;
        {
            std::lock_guard<std::mutex> lock(g_prof_mu);
            on = g_prof_on;
        }
        if (!on) return;
        if (cudaEventCreate(&a) != cudaSuccess || cudaEventCreate(&b) != cudaSuccess) {
            cudaGetLastError();
            a = b = nullptr;
            return;
        }
        cudaEventRecord(a, s);
    }
    ~ProfileScope() {
        if (!a) return;
        cudaEventRecord(b, s);
        std::lock_guard<std::mutex> lock(g_prof_mu);
        g_prof_pending.push_back(EventPair{a, b, kernel});
    }
};

// Bump allocator over one stream-ordered device allocation.
struct Carve {
    char* base = nullptr;
    size_t off = 0;
    size_t size = 0;
    template <class T>
    T* take(size_t count) {
        off = (off + 255) & ~static_cast<size_t>(255);
        T* p = reinterpret_cast<T*>(base + off);
        off += count * sizeof(T);
        return p;
    }
};

template <class T>
size_t bytes_of(size_t count) {
    return ((count * sizeof(T)) + 255) & ~static_cast<size_t>(255);
}

struct StreamBuffer {
    void* ptr = nullptr;
    cudaStream_t stream = nullptr;
    StreamBuffer(size_t bytes, cudaStream_t s) : stream(s) {
        check_cuda(cudaMallocAsync(&ptr, bytes == 0 ? 256 : bytes, s), "cudaMallocAsync(workspace)");
    }
    ~StreamBuffer() {
        if (ptr) cudaFreeAsync(ptr, stream);
    }
    StreamBuffer(const StreamBuffer&) = delete;
    StreamBuffer& operator=(const StreamBuffer&) = delete;
};

}  // namespace

void profile_enable(bool on) {
    std::lock_guard<std::mutex> lock(g_prof_mu);
    g_prof_on = on;
}

void profile_reset() {
    std::lock_guard<std::mutex> lock(g_prof_mu);
    prof_drain_locked();
    for (int i = 0; i < kProfiledKernels; ++i) {
        g_prof_ms[i] = 0.0;
        g_prof_n[i] = 0;
    }
}

void profile_read(int kernel, double* total_ms, long long* launches) {
    std::lock_guard<std::mutex> lock(g_prof_mu);
    prof_drain_locked();
    if (kernel < 0 || kernel >= kProfiledKernels) {
        *total_ms = 0.0;
        *launches = 0;
        return;
    }
    *total_ms = g_prof_ms[kernel];
    *launches = g_prof_n[kernel];
}

void decode(const Options& opt, const float* d_x, int V, const std::vector<ExampleSpec>& ex,
            const CallConstraints& cons, const Outputs& out, const Layout& layout, bool pool,
            bool weights, cudaStream_t stream, DecodeStats* stats, bool synchronize) {
    const int B = static_cast<int>(ex.size());
    if (B <= 0) return;
    const bool dynamic = cons.repetition_penalty > 1.0f || cons.no_repeat_ngram > 0;

    std::vector<dbs_dev::ExampleDesc> desc(B);
    std::vector<int64_t> row_prefix(B + 1, 0);
    int max_T = 0, max_K = 0, max_C = 0, max_N = 0, max_P = 0;
    int64_t rows = 0, list_entries = 0;
    for (int b = 0; b < B; ++b) {
        const ExampleSpec& e = ex[b];
        const int P = layout.P[b];
        const int N = pool ? P : e.K;
        int slack = 0;
        if (dynamic) slack = 8 + N / 8;
        const int C = N + slack;
        if (static_cast<int64_t>(e.K) * C > dbs_dev::kMaxMergeCandidates) {
            throw LengthError("beam_size * relaxed pool exceeds the per-step merge capacity of " +
                              std::to_string(dbs_dev::kMaxMergeCandidates) + " candidates");
        }
        if (e.K > 1024) throw LengthError("beam_size above 1024 is not supported by the device decoder");
        dbs_dev::ExampleDesc& d = desc[b];
        d.x_offset = e.x_offset;
        d.row_begin = rows;
        d.list_offset = list_entries;
        d.sel_offset = layout.sel_offset[b];
        d.pool_offset = layout.pool_offset[b];
        d.final_offset = layout.final_offset[b];
        d.grad_offset = layout.grad_offset[b];
        d.sparse_offset = layout.sparse_offset[b];
        d.T = e.T;
        d.K = e.K;
        d.k_stride = e.k_stride;
        d.P = P;
        d.N = N;
        d.C = C;
        d.sel_stride = e.K;
        d.pool_stride = P;
        d.sel_t_stride = e.K;
        d.pool_t_stride = P;
        d.eos = e.eos;
        d.min_length = e.min_length;
        d.banned = e.banned;
        d.forced = e.forced;
        rows += static_cast<int64_t>(e.T) * e.K;
        list_entries += static_cast<int64_t>(e.T) * e.K * C;
        row_prefix[b + 1] = rows;
        max_T = std::max(max_T, e.T);
        max_K = std::max(max_K, e.K);
        max_C = std::max(max_C, C);
        max_N = std::max(max_N, N);
        max_P = std::max(max_P, P);
    }
    if (pool && out.relaxed_weights && max_P > 1024) {
        throw LengthError("relaxed pool above 1024 entries is not supported by the device decoder");
    }
    const int lmax = max_T + 1;
    std::vector<float> pen, inv;
    penalty_tables(opt.length_penalty_alpha, lmax, pen, inv);

    size_t ws = 0;
    ws += bytes_of<dbs_dev::ExampleDesc>(B);
    ws += bytes_of<int64_t>(B + 1);
    ws += 2 * bytes_of<float>(lmax + 1);
    ws += bytes_of<uint64_t>(static_cast<size_t>(list_entries));
    ws += bytes_of<int32_t>(static_cast<size_t>(rows));
    ws += bytes_of<float>(static_cast<size_t>(rows));
    ws += bytes_of<int32_t>(B);
    ws += bytes_of<unsigned long long>(4);
    if (dynamic) ws += bytes_of<int32_t>(static_cast<size_t>(B) * 3 * max_K * max_T);
    StreamBuffer buf(ws, stream);
    Carve cv{static_cast<char*>(buf.ptr), 0, ws};

    dbs_dev::DecodeParams p{};
    auto* d_desc = cv.take<dbs_dev::ExampleDesc>(B);
    auto* d_prefix = cv.take<int64_t>(B + 1);
    auto* d_pen = cv.take<float>(lmax + 1);
    auto* d_inv = cv.take<float>(lmax + 1);
    p.lists = cv.take<uint64_t>(static_cast<size_t>(list_entries));
    p.list_count = cv.take<int32_t>(static_cast<size_t>(rows));
    p.list_bound = cv.take<float>(static_cast<size_t>(rows));
    p.status = cv.take<int32_t>(B);
    p.counters = cv.take<unsigned long long>(4);
    p.seq_scratch = dynamic ? cv.take<int32_t>(static_cast<size_t>(B) * 3 * max_K * max_T) : nullptr;

    check_cuda(cudaMemcpyAsync(d_desc, desc.data(), sizeof(dbs_dev::ExampleDesc) * B, cudaMemcpyHostToDevice, stream),
               "upload descriptors");
    check_cuda(cudaMemcpyAsync(d_prefix, row_prefix.data(), sizeof(int64_t) * (B + 1), cudaMemcpyHostToDevice, stream),
               "upload row prefix");
    check_cuda(cudaMemcpyAsync(d_pen, pen.data(), sizeof(float) * (lmax + 1), cudaMemcpyHostToDevice, stream),
               "upload penalty table");
    check_cuda(cudaMemcpyAsync(d_inv, inv.data(), sizeof(float) * (lmax + 1), cudaMemcpyHostToDevice, stream),
               "upload penalty table");
    check_cuda(cudaMemsetAsync(p.status, 0, sizeof(int32_t) * B, stream), "clear status");
    check_cuda(cudaMemsetAsync(p.counters, 0, sizeof(unsigned long long) * 4, stream), "clear counters");

    p.x = d_x;
    p.V = V;
    p.B = B;
    p.total_rows = rows;
    p.desc = d_desc;
    p.row_prefix = d_prefix;
    p.pen = d_pen;
    p.inv_pen = d_inv;
    p.Lmax = lmax;
    p.selected_temperature = opt.selected_temperature;
    p.soft_topk_temperature = opt.soft_topk_temperature;
    p.soft_topk_tolerance = opt.soft_topk_tolerance;
    p.soft_topk_max_iters = opt.soft_topk_max_iters;
    p.repetition_penalty = cons.repetition_penalty;
    p.log_repetition_penalty = cons.repetition_penalty > 1.0f ? std::log(cons.repetition_penalty) : 0.0f;
    p.no_repeat_ngram = cons.no_repeat_ngram;
    p.validate_inputs = opt.validate_inputs;
    p.parents = out.parents;
    p.tokens = out.tokens;
    p.lengths = out.lengths;
    p.raw_scores = out.raw_scores;
    p.scores = out.scores;
    p.weights = weights ? out.weights : nullptr;
    p.from_logprob = out.from_logprob;
    if (pool) {
        p.pool_parents = out.pool_parents;
        p.pool_tokens = out.pool_tokens;
        p.pool_lengths = out.pool_lengths;
        p.pool_raw_scores = out.pool_raw_scores;
        p.pool_scores = out.pool_scores;
        p.relaxed_weights = out.relaxed_weights;
        p.pool_from_logprob = out.pool_from_logprob;
    }
    p.final_raw_scores = out.final_raw_scores;
    p.final_scores = out.final_scores;

    if (opt.validate_inputs) {
        ProfileScope ps(kValidate, stream);
        check_cuda(dbs_dev::launch_validate(p, stream), "validate kernel");
    }
    {
        ProfileScope ps(kRowScan, stream);
        check_cuda(dbs_dev::launch_row_scan(p, max_C, device_sm_count(), stream), "row scan kernel");
    }
    {
        ProfileScope ps(kStepMerge, stream);
        check_cuda(dbs_dev::launch_step_merge(p, max_K, max_C, max_T, max_N, dynamic, stream), "step merge kernel");
    }
    const bool want_w = (p.weights && p.scores) || (p.relaxed_weights && p.pool_scores);
    if (want_w) {
        ProfileScope ps(kWeights, stream);
        check_cuda(dbs_dev::launch_weights(p, max_T, max_K, max_P, stream), "weights kernel");
    }

    if (synchronize) {
        std::vector<int32_t> status(B, 0);
        unsigned long long counters[4] = {0, 0, 0, 0};
        check_cuda(cudaMemcpyAsync(status.data(), p.status, sizeof(int32_t) * B, cudaMemcpyDeviceToHost, stream),
                   "read status");
        check_cuda(cudaMemcpyAsync(counters, p.counters, sizeof(counters), cudaMemcpyDeviceToHost, stream),
                   "read counters");
        check_cuda(cudaStreamSynchronize(stream), "decode");
        if (stats) {
            stats->row_rescans = counters[0];
            stats->merge_fallbacks = counters[1];
        }
        if (opt.validate_inputs) {
            for (int b = 0; b < B; ++b)
                if (status[b]) throw InvalidArgument("log_probs contains NaN or +Inf");
        }
    }
}

void backward(const Options& opt, int V, const std::vector<ExampleSpec>& ex, const Layout& layout,
              const BackwardInputs& in, const BackwardOutputs& out, cudaStream_t stream, bool zero_dense) {
    const int B = static_cast<int>(ex.size());
    if (B <= 0) return;
    std::vector<dbs_dev::ExampleDesc> desc(B);
    int max_T = 0, max_K = 0, max_P = 0;
    for (int b = 0; b < B; ++b) {
        const ExampleSpec& e = ex[b];
        dbs_dev::ExampleDesc& d = desc[b];
        std::memset(&d, 0, sizeof(d));
        d.T = e.T;
        d.K = e.K;
        d.P = layout.P[b];
        d.sel_offset = layout.sel_offset[b];
        d.pool_offset = layout.pool_offset[b];
        d.final_offset = layout.final_offset[b];
        d.grad_offset = layout.grad_offset[b];
        d.sparse_offset = layout.sparse_offset[b];
        d.sel_t_stride = e.K;
        d.pool_t_stride = d.P;
        max_T = std::max(max_T, e.T);
        max_K = std::max(max_K, e.K);
        max_P = std::max(max_P, d.P);
    }
    if (max_K + max_P > 4096) throw LengthError("beam_size + relaxed pool above 4096 per step is not supported by the device backward");
    const int lmax = max_T + 1;
    std::vector<float> pen, inv;
    penalty_tables(opt.length_penalty_alpha, lmax, pen, inv);
    const bool sparse = out.sparse_indices != nullptr;
    size_t ws = bytes_of<dbs_dev::ExampleDesc>(B) + bytes_of<float>(lmax + 1) +
                bytes_of<int32_t>(static_cast<size_t>(B) * max_T);
    StreamBuffer buf(ws, stream);
    Carve cv{static_cast<char*>(buf.ptr), 0, ws};
    auto* d_desc = cv.take<dbs_dev::ExampleDesc>(B);
    auto* d_inv = cv.take<float>(lmax + 1);
    auto* d_steps = cv.take<int32_t>(static_cast<size_t>(B) * max_T);
    check_cuda(cudaMemcpyAsync(d_desc, desc.data(), sizeof(dbs_dev::ExampleDesc) * B, cudaMemcpyHostToDevice, stream),
               "upload descriptors");
    check_cuda(cudaMemcpyAsync(d_inv, inv.data(), sizeof(float) * (lmax + 1), cudaMemcpyHostToDevice, stream),
               "upload penalty table");
    if (!sparse && out.grad_dense && zero_dense) {
        ProfileScope ps(kFillZero, stream);
        check_cuda(dbs_dev::launch_fill_zero(out.grad_dense, layout.grad_total, device_sm_count(), stream),
                   "zero fill kernel");
    }
    dbs_dev::BackwardParams p{};
    p.V = V;
    p.B = B;
    p.max_T = max_T;
    p.desc = d_desc;
    p.inv_pen = d_inv;
    p.Lmax = lmax;
    p.selected_temperature = opt.selected_temperature;
    p.soft_topk_temperature = opt.soft_topk_temperature;
    p.parents = in.parents;
    p.tokens = in.tokens;
    p.lengths = in.lengths;
    p.weights = in.weights;
    p.from_logprob = in.from_logprob;
    p.pool_parents = in.pool_parents;
    p.pool_tokens = in.pool_tokens;
    p.pool_lengths = in.pool_lengths;
    p.relaxed_weights = in.relaxed_weights;
    p.pool_from_logprob = in.pool_from_logprob;
    p.grad_selected = in.grad_selected;
    p.grad_relaxed = in.grad_relaxed;
    p.grad_final = in.grad_final;
    p.grad_dense = out.grad_dense;
    p.sparse_indices = out.sparse_indices;
    p.sparse_values = out.sparse_values;
    p.sparse_counts = out.sparse_counts;
    p.step_counts = d_steps;
    p.grad_initial = out.grad_initial;
    ProfileScope ps(kBackward, stream);
    check_cuda(dbs_dev::launch_backward(p, max_K, max_P, sparse, stream), "backward kernel");
}

}  // namespace dbs_host
