// C ABI of libdbs.so (include/dbs.h, include/dbs_device.h) over the device
// engine. The handle / result / error / stats contract follows the
// reference's C ABI layer (src/differentiable_beam.cpp:3049-4210); the
// decode and backward themselves always run as device kernels.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <limits>
#include <memory>
#include <mutex>
#include <new>
#include <stdexcept>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "dbs.h"
#include "dbs_device.h"
#include "engine.h"

using dbs_host::CallConstraints;
using dbs_host::ExampleSpec;
using dbs_host::InvalidArgument;
using dbs_host::Layout;
using dbs_host::Options;

namespace {

std::atomic<int64_t> g_alloc_calls{0};
std::atomic<int64_t> g_alloc_bytes{0};
thread_local std::string g_last_error;

constexpr int kKernelCuda = 5;

int64_t now_ns() {
    return std::chrono::duration_cast<std::chrono::nanoseconds>(
               std::chrono::steady_clock::now().time_since_epoch())
        .count();
}

size_t checked_mul(size_t a, size_t b, const char* what) {
    if (a != 0 && b > std::numeric_limits<size_t>::max() / a) throw std::overflow_error(what);
    return a * b;
}

// Device allocation owned by one call, released in stream order.
struct DeviceBuffer {
    void* ptr = nullptr;
    size_t bytes = 0;
    cudaStream_t stream = nullptr;
    DeviceBuffer() = default;
    DeviceBuffer(size_t n, cudaStream_t s) : bytes(n), stream(s) {
        if (n == 0) return;
        cudaError_t err = cudaMallocAsync(&ptr, n, s);
        if (err != cudaSuccess) {
            ptr = nullptr;
            if (err == cudaErrorMemoryAllocation) throw std::bad_alloc();
            dbs_host::check_cuda(err, "cudaMallocAsync");
        }
        g_alloc_calls.fetch_add(1, std::memory_order_relaxed);
        g_alloc_bytes.fetch_add(static_cast<int64_t>(n), std::memory_order_relaxed);
    }
    ~DeviceBuffer() {
        if (ptr) {
            cudaFreeAsync(ptr, stream);
            g_alloc_bytes.fetch_sub(static_cast<int64_t>(bytes), std::memory_order_relaxed);
        }
    }
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    template <class T>
    T* as() const { return static_cast<T*>(ptr); }
};

template <class T>
void host_alloc(std::vector<T>& v, size_t n, T fill) {
    v.assign(n, fill);
    g_alloc_calls.fetch_add(1, std::memory_order_relaxed);
    g_alloc_bytes.fetch_add(static_cast<int64_t>(n * sizeof(T)), std::memory_order_relaxed);
}

bool is_device_pointer(const void* p) {
    if (!p) return false;
    cudaPointerAttributes a{};
    cudaError_t err = cudaPointerGetAttributes(&a, p);
    if (err != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// Stream of one host-pointer ABI call: a private stream created blocking, so
// it is ordered after pending work on the legacy default stream; the call
// waits for it before returning. The device entry points never use this:
// they run on the caller's stream verbatim (NULL = legacy default stream).
struct CallStream {
    cudaStream_t s = nullptr;
    explicit CallStream(void*) {
        dbs_host::check_cuda(cudaStreamCreate(&s), "cudaStreamCreate");
    }
    ~CallStream() {
        cudaStreamSynchronize(s);
        cudaStreamDestroy(s);
    }
};

// A calling thread's stream and pinned staging buffer on the current device,
// kept for the thread's later calls: the per-example host-buffer backward
// moves a few small arrays each way, and a stream created per call or a
// pageable copy per array cost more than the kernel. Never freed (the
// process may outlive the CUDA runtime's own teardown order).
struct ThreadStaging {
    int device = -1;
    cudaStream_t s = nullptr;
    char* pinned = nullptr;
    size_t bytes = 0;
};
ThreadStaging& thread_staging(size_t need) {
    thread_local std::vector<ThreadStaging> per_device;
    int dev = 0;
    dbs_host::check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    ThreadStaging* t = nullptr;
    for (ThreadStaging& c : per_device)
        if (c.device == dev) t = &c;
    if (!t) {
        per_device.push_back(ThreadStaging{});
        t = &per_device.back();
        t->device = dev;
        dbs_host::check_cuda(cudaStreamCreateWithFlags(&t->s, cudaStreamNonBlocking), "cudaStreamCreate");
    }
    if (t->bytes < need) {
        if (t->pinned) dbs_host::check_cuda(cudaFreeHost(t->pinned), "cudaFreeHost(staging)");
        t->pinned = nullptr;
        t->bytes = 0;
        const size_t n = std::max(need + need / 4, static_cast<size_t>(64) << 10);
        dbs_host::check_cuda(cudaHostAlloc(reinterpret_cast<void**>(&t->pinned), n, cudaHostAllocDefault),
                             "cudaHostAlloc(staging)");
        t->bytes = n;
    }
    return *t;
}

}  // namespace

// ---------------------------------------------------------------------------
// Handle types
// ---------------------------------------------------------------------------
struct DBSDecoderHandle {
    Options options;
    int beam_size = 0;
    std::mutex error_mutex;
    std::string last_error;
    std::mutex stats_mutex;
    DBSStatsC stats{};
    uint64_t deterministic_seed = 0;
};

struct ExampleInfo {
    int T = 0, K = 0, P = 0, V = 0, eos = -1;
    int64_t sel = 0, pool = 0, fin = 0;
};

// Host mirror of one decode call (one or more examples, tight layout).
struct ResultStore {
    Options opt;
    int V = 0;
    std::vector<ExampleInfo> ex;
    std::vector<int32_t> parents, tokens, lengths, pool_parents, pool_tokens, pool_lengths;
    std::vector<float> raw, scores, weights, pool_raw, pool_scores, relaxed, final_raw, final_scores;
    std::vector<uint8_t> flp, pool_flp;
};

struct DBSResultHandle {
    std::shared_ptr<ResultStore> store;
    int index = 0;
    const ExampleInfo& info() const { return store->ex[static_cast<size_t>(index)]; }
};

struct DBSBatchResultHandle {
    std::shared_ptr<ResultStore> store;
    std::vector<DBSResultHandle> items;
};

struct DBSBackwardHandle {
    std::vector<float> grad_log_probs;
    std::vector<float> grad_initial;
    std::vector<int64_t> indices;
    std::vector<float> values;
    bool sparse = false;
};

struct DBSWorkspaceHandle {
    std::mutex mutex;
    std::vector<float> f32;
    std::vector<int32_t> i32;
};

// ---------------------------------------------------------------------------
// Error and stats plumbing (src/differentiable_beam.cpp:3078-3143)
// ---------------------------------------------------------------------------
namespace {

void set_error(DBSDecoderHandle* h, const std::string& msg) {
    g_last_error = msg;
    if (h) {
        std::lock_guard<std::mutex> lock(h->error_mutex);
        h->last_error = msg;
    }
}

void clear_error(DBSDecoderHandle* h) {
    g_last_error.clear();
    if (h) {
        std::lock_guard<std::mutex> lock(h->error_mutex);
        h->last_error.clear();
    }
}

int classify(const std::exception& e) {
    if (dynamic_cast<const std::invalid_argument*>(&e)) return 1;
    if (dynamic_cast<const std::bad_alloc*>(&e)) return 3;
    if (dynamic_cast<const std::overflow_error*>(&e)) return 4;
    if (dynamic_cast<const std::length_error*>(&e)) return 4;
    return 2;
}

void mark_error(DBSDecoderHandle* h, int category) {
    if (!h) return;
    std::lock_guard<std::mutex> lock(h->stats_mutex);
    h->stats.last_error_category = category;
}

void record_decode(DBSDecoderHandle* h, const ExampleInfo& r, int64_t ns, int threads, bool model_step) {
    if (!h) return;
    std::lock_guard<std::mutex> lock(h->stats_mutex);
    h->stats.abi_version = DBS_ABI_VERSION;
    h->stats.last_kernel = kKernelCuda;
    h->stats.used_batch_threads = threads;
    h->stats.used_model_step_callback = model_step ? 1 : 0;
    h->stats.last_decode_ns = ns;
    h->stats.last_selected_count = static_cast<int64_t>(r.T) * r.K;
    h->stats.last_pool_count = static_cast<int64_t>(r.T) * r.P;
    h->stats.last_logprob_count = static_cast<int64_t>(r.T) * r.K * r.V;
    h->stats.last_allocation_bytes = static_cast<int64_t>(r.T) * r.K * (4 + 4 + 4 + 4) +
                                     static_cast<int64_t>(r.T) * r.P * (4 + 4 + 4);
    h->stats.last_error_category = 0;
}

void record_backward(DBSDecoderHandle* h, const DBSBackwardHandle& b, int64_t ns) {
    if (!h) return;
    std::lock_guard<std::mutex> lock(h->stats_mutex);
    h->stats.abi_version = DBS_ABI_VERSION;
    h->stats.used_sparse_backward = b.sparse ? 1 : 0;
    h->stats.used_dense_backward = b.sparse ? 0 : 1;
    h->stats.last_backward_ns = ns;
    h->stats.last_sparse_grad_count = static_cast<int64_t>(b.values.size());
    h->stats.last_error_category = 0;
}

// from_c_options (src/differentiable_beam.cpp:3145-3177) and the decoder
// constructor's checks and clamps (:1390-1426).
Options parse_options(const DBSOptionsC& c) {
    Options o;
    o.beam_size = c.beam_size > 0 ? c.beam_size : 8;
    o.eos_token = c.eos_token;
    o.selected_temperature = c.selected_temperature > 0.0f ? c.selected_temperature : 1.0f;
    o.soft_topk_temperature = c.soft_topk_temperature > 0.0f ? c.soft_topk_temperature : 0.25f;
    o.relaxed_pool_multiplier = c.relaxed_pool_multiplier > 0 ? c.relaxed_pool_multiplier : 8;
    o.vocab_block = c.vocab_block > 0 ? c.vocab_block : 4096;
    o.length_penalty_alpha = c.length_penalty_alpha >= 0.0f ? c.length_penalty_alpha : 0.0f;
    o.soft_topk_tolerance = c.soft_topk_tolerance > 0.0f ? c.soft_topk_tolerance : 1.0e-4f;
    o.soft_topk_max_iters = c.soft_topk_max_iters > 0 ? c.soft_topk_max_iters : 48;
    o.min_length = c.min_length >= 0 ? c.min_length : 0;
    o.validate_inputs = c.validate_inputs == 0 ? 0 : 1;
    o.max_dense_gradient_elements =
        c.max_dense_gradient_elements > 0 ? c.max_dense_gradient_elements : 100000000LL;
    return o;
}

void check_options(Options& o) {
    if (o.beam_size <= 0) throw std::invalid_argument("beam_size must be positive");
    if (!(o.selected_temperature > 0.0f)) throw std::invalid_argument("selected_temperature must be positive");
    if (!(o.soft_topk_temperature > 0.0f)) throw std::invalid_argument("soft_topk_temperature must be positive");
    if (o.soft_topk_max_iters <= 0) throw std::invalid_argument("soft_topk_max_iters must be positive");
    if (!(o.soft_topk_tolerance > 0.0f)) throw std::invalid_argument("soft_topk_tolerance must be positive");
    if (o.length_penalty_alpha < 0.0f) throw std::invalid_argument("length_penalty_alpha cannot be negative");
    if (o.min_length < 0) throw std::invalid_argument("min_length cannot be negative");
    if (o.max_dense_gradient_elements <= 0)
        throw std::invalid_argument("max_dense_gradient_elements must be positive");
    o.vocab_block = std::max(16, o.vocab_block);
    o.relaxed_pool_multiplier = std::max(1, o.relaxed_pool_multiplier);
}

// Host-side description of one example before staging.
struct HostExample {
    int T = 0;
    int K = 0;
    int eos = -1;
    int min_length = 0;
    int64_t x_offset = 0;   // element offset in the caller's array
    int k_stride = 0;       // rows per step in the caller's array
    const uint8_t* banned = nullptr;  // caller pointer [V] (host or device)
    const int32_t* forced = nullptr;  // caller pointer [>=T] (host or device)
};

// Argument checks of decode_constrained (src/differentiable_beam.cpp:1433-1464)
// for one example; `forced` must be readable on the host here.
void check_example(const Options& opt, const float* x, int T, int V, int K, int eos,
                   const int32_t* forced_host) {
    if (!x) throw std::invalid_argument("log_probs cannot be null");
    if (T <= 0) throw std::invalid_argument("steps must be positive");
    if (V <= 0) throw std::invalid_argument("vocab_size must be positive");
    if (eos >= V) throw std::invalid_argument("eos_token is outside vocab");
    if (forced_host) {
        for (int t = 0; t < T; ++t)
            if (forced_host[t] >= V) throw std::invalid_argument("forced token is outside vocab");
    }
    const int P = dbs_host::pool_size(K, opt.relaxed_pool_multiplier);
    const size_t sel = checked_mul(static_cast<size_t>(T), static_cast<size_t>(K), "selected result size overflow");
    (void)checked_mul(static_cast<size_t>(T), static_cast<size_t>(P), "pool result size overflow");
    (void)checked_mul(sel, static_cast<size_t>(V), "log-prob tensor size overflow");
}

// Bytes of host log-probs staged on the device per chunk. Two chunks are in
// flight (one decoding while the next is copied), so chunks stay a few GB:
// the copies then run back to back at the host link's rate.
size_t device_budget_bytes() {
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) {
        cudaGetLastError();
        return static_cast<size_t>(1) << 30;
    }
    size_t b = free_b / 8;
    const size_t cap = static_cast<size_t>(4) << 30;
    return std::min(b, cap);
}

// Runs the device decode of `hx` over the caller array x (host or device) and
// returns the host mirror. Host inputs are staged in example chunks that fit
// half of the free device memory; each example is packed tight [T,K,V].
// Reads a caller array that may live on the device into host memory.
template <class T>
std::vector<T> host_copy(const T* p, size_t n) {
    std::vector<T> v(n);
    if (n == 0 || !p) return v;
    if (is_device_pointer(p)) {
        dbs_host::check_cuda(cudaMemcpy(v.data(), p, n * sizeof(T), cudaMemcpyDeviceToHost), "read caller array");
    } else {
        std::memcpy(v.data(), p, n * sizeof(T));
    }
    return v;
}

std::shared_ptr<ResultStore> run_decode(DBSDecoderHandle* h, const Options& opt, const float* x, int V,
                                        const std::vector<HostExample>& hx, const CallConstraints& cons,
                                        DBSDecoderHandle* stats_handle,
                                        const dbs_host::TokenFilter* filter = nullptr,
                                        const uint16_t* x16 = nullptr, bool x16_bf16 = false,
                                        const dbs_host::StepRows* rows = nullptr) {
    auto store = std::make_shared<ResultStore>();
    store->opt = opt;
    store->V = V;
    const int B = static_cast<int>(hx.size());
    store->ex.resize(B);
    std::vector<ExampleSpec> all(B);
    for (int b = 0; b < B; ++b) {
        all[b].T = hx[b].T;
        all[b].K = hx[b].K;
        all[b].eos = hx[b].eos;
        all[b].min_length = hx[b].min_length;
    }
    const Layout L = dbs_host::make_layout(opt, all, V);
    for (int b = 0; b < B; ++b) {
        ExampleInfo& e = store->ex[b];
        e.T = hx[b].T;
        e.K = hx[b].K;
        e.P = L.P[b];
        e.V = V;
        e.eos = hx[b].eos;
        e.sel = L.sel_offset[b];
        e.pool = L.pool_offset[b];
        e.fin = L.final_offset[b];
    }
    host_alloc(store->parents, L.sel_total, int32_t{-1});
    host_alloc(store->tokens, L.sel_total, int32_t{-1});
    host_alloc(store->lengths, L.sel_total, int32_t{0});
    host_alloc(store->raw, L.sel_total, -std::numeric_limits<float>::infinity());
    host_alloc(store->scores, L.sel_total, -std::numeric_limits<float>::infinity());
    host_alloc(store->weights, L.sel_total, 0.0f);
    host_alloc(store->flp, L.sel_total, uint8_t{0});
    host_alloc(store->pool_parents, L.pool_total, int32_t{-1});
    host_alloc(store->pool_tokens, L.pool_total, int32_t{-1});
    host_alloc(store->pool_lengths, L.pool_total, int32_t{0});
    host_alloc(store->pool_raw, L.pool_total, -std::numeric_limits<float>::infinity());
    host_alloc(store->pool_scores, L.pool_total, -std::numeric_limits<float>::infinity());
    host_alloc(store->relaxed, L.pool_total, 0.0f);
    host_alloc(store->pool_flp, L.pool_total, uint8_t{0});
    host_alloc(store->final_raw, L.final_total, -std::numeric_limits<float>::infinity());
    host_alloc(store->final_scores, L.final_total, -std::numeric_limits<float>::infinity());

    CallStream cs(nullptr);
    cudaStream_t s = cs.s;
    // 16-bit inputs arrive on the device; model-step rows are produced there
    const bool x_dev = x16 != nullptr || rows != nullptr || is_device_pointer(x);
    const size_t budget = device_budget_bytes();
    // Example chunks: host inputs are staged a chunk at a time into one of
    // two device buffers; the next chunk's copy (on a copy stream) runs while
    // the current chunk decodes and its results are read back.
    struct Chunk {
        int b0, b1;
        int64_t elems;
    };
    std::vector<Chunk> chunks;
    int64_t max_elems = 0;
    for (int c0 = 0; c0 < B;) {
        int c1 = c0;
        size_t bytes = 0;
        int64_t elems = 0;
        while (c1 < B) {
            const int64_t ne = x_dev ? 0 : static_cast<int64_t>(hx[c1].T) * hx[c1].K * V;
            const size_t need = static_cast<size_t>(ne) * sizeof(float);
            if (c1 > c0 && bytes + need > budget) break;
            bytes += need;
            elems += ne;
            ++c1;
        }
        chunks.push_back(Chunk{c0, c1, elems});
        max_elems = std::max(max_elems, elems);
        c0 = c1;
    }
    const int n_staged = x_dev ? 0 : (chunks.size() > 1 ? 2 : 1);
    std::unique_ptr<DeviceBuffer> stage_buf[2];
    for (int i = 0; i < n_staged; ++i)
        stage_buf[i].reset(new DeviceBuffer(static_cast<size_t>(max_elems) * sizeof(float), s));
    std::unique_ptr<CallStream> copy_cs;
    cudaEvent_t staged_ev[2] = {nullptr, nullptr};
    struct EventPairGuard {
        cudaEvent_t* e;
        ~EventPairGuard() {
            for (int i = 0; i < 2; ++i)
                if (e[i]) cudaEventDestroy(e[i]);
        }
    } staged_guard{staged_ev};
    if (n_staged) {
        copy_cs.reset(new CallStream(nullptr));
        // the staging buffers come from `s`'s allocations: the copy stream waits for them
        for (int i = 0; i < 2; ++i)
            dbs_host::check_cuda(cudaEventCreateWithFlags(&staged_ev[i], cudaEventDisableTiming), "cudaEventCreate");
        dbs_host::check_cuda(cudaEventRecord(staged_ev[0], s), "cudaEventRecord");
        dbs_host::check_cuda(cudaStreamWaitEvent(copy_cs->s, staged_ev[0], 0), "cudaStreamWaitEvent");
    }
    auto stage = [&](size_t ci) {   // host -> device copy of chunk ci's log-probs
        const Chunk& c = chunks[ci];
        float* dst = stage_buf[ci & 1]->as<float>();
        // examples stored back to back without padding beams: one copy
        bool packed = true;
        for (int b = c.b0; b < c.b1 && packed; ++b) {
            const HostExample& e = hx[b];
            packed = e.k_stride == e.K && (b == c.b0 || e.x_offset == hx[b - 1].x_offset +
                                                             static_cast<int64_t>(hx[b - 1].T) * hx[b - 1].k_stride * V);
        }
        if (packed) {
            dbs_host::check_cuda(cudaMemcpyAsync(dst, x + hx[c.b0].x_offset, static_cast<size_t>(c.elems) * sizeof(float),
                                                 cudaMemcpyHostToDevice, copy_cs->s),
                                 "stage log_probs");
            dbs_host::check_cuda(cudaEventRecord(staged_ev[ci & 1], copy_cs->s), "cudaEventRecord");
            return;
        }
        int64_t off = 0;
        for (int b = c.b0; b < c.b1; ++b) {
            const HostExample& e = hx[b];
            const size_t width = static_cast<size_t>(e.K) * V * sizeof(float);
            const size_t pitch = static_cast<size_t>(e.k_stride) * V * sizeof(float);
            dbs_host::check_cuda(cudaMemcpy2DAsync(dst + off, width, x + e.x_offset, pitch, width,
                                                   static_cast<size_t>(e.T), cudaMemcpyHostToDevice, copy_cs->s),
                                 "stage log_probs");
            off += static_cast<int64_t>(e.T) * e.K * V;
        }
        dbs_host::check_cuda(cudaEventRecord(staged_ev[ci & 1], copy_cs->s), "cudaEventRecord");
    };
    if (n_staged) stage(0);
    for (size_t ci = 0; ci < chunks.size(); ++ci) {
        const int b0 = chunks[ci].b0, b1 = chunks[ci].b1;
        // the next chunk's buffer was last read by chunk ci - 1, whose decode
        // has finished (each chunk's decode synchronises below)
        if (n_staged && ci + 1 < chunks.size()) stage(ci + 1);
        if (n_staged) dbs_host::check_cuda(cudaStreamWaitEvent(s, staged_ev[ci & 1], 0), "cudaStreamWaitEvent");
        const int nb = b1 - b0;
        std::vector<ExampleSpec> spec(nb);
        int64_t staged_elems = 0;
        for (int i = 0; i < nb; ++i) {
            const HostExample& e = hx[b0 + i];
            spec[i].T = e.T;
            spec[i].K = e.K;
            spec[i].eos = e.eos;
            spec[i].min_length = e.min_length;
            if (x_dev) {
                spec[i].x_offset = e.x_offset;
                spec[i].k_stride = e.k_stride;
            } else {
                spec[i].x_offset = staged_elems;
                spec[i].k_stride = e.K;
                staged_elems += static_cast<int64_t>(e.T) * e.K * V;
            }
        }
        // constraint arrays
        std::vector<std::unique_ptr<DeviceBuffer>> cbufs;
        for (int i = 0; i < nb; ++i) {
            const HostExample& e = hx[b0 + i];
            if (e.banned) {
                if (is_device_pointer(e.banned)) {
                    spec[i].banned = e.banned;
                } else {
                    cbufs.emplace_back(new DeviceBuffer(static_cast<size_t>(V), s));
                    dbs_host::check_cuda(cudaMemcpyAsync(cbufs.back()->ptr, e.banned, V, cudaMemcpyHostToDevice, s),
                                         "stage banned tokens");
                    spec[i].banned = cbufs.back()->as<uint8_t>();
                }
            }
            if (e.forced) {
                if (is_device_pointer(e.forced)) {
                    spec[i].forced = e.forced;
                } else {
                    cbufs.emplace_back(new DeviceBuffer(sizeof(int32_t) * e.T, s));
                    dbs_host::check_cuda(cudaMemcpyAsync(cbufs.back()->ptr, e.forced, sizeof(int32_t) * e.T,
                                                         cudaMemcpyHostToDevice, s),
                                         "stage forced tokens");
                    spec[i].forced = cbufs.back()->as<int32_t>();
                }
            }
        }
        const Layout CL = dbs_host::make_layout(opt, spec, V);
        const size_t nsel = CL.sel_total, npool = CL.pool_total, nfin = CL.final_total;
        DeviceBuffer ob(nsel * (3 * 4 + 3 * 4 + 1) + npool * (3 * 4 + 3 * 4 + 1) + nfin * 8 + 64 * 16, s);
        char* cur = ob.as<char>();
        auto take = [&](size_t bytes_needed) {
            char* p = cur;
            cur += (bytes_needed + 15) & ~static_cast<size_t>(15);
            return p;
        };
        dbs_host::Outputs o;
        o.parents = reinterpret_cast<int32_t*>(take(nsel * 4));
        o.tokens = reinterpret_cast<int32_t*>(take(nsel * 4));
        o.lengths = reinterpret_cast<int32_t*>(take(nsel * 4));
        o.raw_scores = reinterpret_cast<float*>(take(nsel * 4));
        o.scores = reinterpret_cast<float*>(take(nsel * 4));
        o.weights = reinterpret_cast<float*>(take(nsel * 4));
        o.from_logprob = reinterpret_cast<uint8_t*>(take(nsel));
        o.pool_parents = reinterpret_cast<int32_t*>(take(npool * 4));
        o.pool_tokens = reinterpret_cast<int32_t*>(take(npool * 4));
        o.pool_lengths = reinterpret_cast<int32_t*>(take(npool * 4));
        o.pool_raw_scores = reinterpret_cast<float*>(take(npool * 4));
        o.pool_scores = reinterpret_cast<float*>(take(npool * 4));
        o.relaxed_weights = reinterpret_cast<float*>(take(npool * 4));
        o.pool_from_logprob = reinterpret_cast<uint8_t*>(take(npool));
        o.final_raw_scores = reinterpret_cast<float*>(take(nfin * 4));
        o.final_scores = reinterpret_cast<float*>(take(nfin * 4));
        const float* dx = x_dev ? x : stage_buf[ci & 1]->as<float>();
        dbs_host::DecodeStats st;
        if (rows) {
            // one example (dbs_decode_model_steps): rows arrive step by step
            DeviceBuffer xr(static_cast<size_t>(spec[0].T) * spec[0].K * V * sizeof(float), s);
            spec[0].x_offset = 0;
            spec[0].k_stride = spec[0].K;
            dbs_host::decode_model_steps(opt, xr.as<float>(), V, spec[0], o, CL, s, &st, *rows);
        } else if (filter) {
            // one example (dbs_decode_constrained_ex): the host checks need the
            // constraint arrays in host memory
            const HostExample& e = hx[b0];
            const std::vector<uint8_t> hb = host_copy(e.banned, e.banned ? static_cast<size_t>(V) : 0);
            const std::vector<int32_t> hf = host_copy(e.forced, e.forced ? static_cast<size_t>(e.T) : 0);
            dbs_host::decode_filtered(opt, dx, V, spec[0], e.banned ? hb.data() : nullptr,
                                      e.forced ? hf.data() : nullptr, cons, o, CL, s, &st, *filter);
        } else {
            dbs_host::DecodeControl ctl;
            ctl.x16 = x16;
            ctl.x16_bf16 = x16_bf16;
            dbs_host::decode(opt, x16 ? nullptr : dx, V, spec, cons, o, CL, true, true, s, &st, ctl);
        }
        const ExampleInfo& first = store->ex[b0];
        const int64_t so = first.sel, po = first.pool, fo = first.fin;
        auto d2h = [&](void* dst, const void* src, size_t n) {
            if (n) dbs_host::check_cuda(cudaMemcpyAsync(dst, src, n, cudaMemcpyDeviceToHost, s), "read results");
        };
        d2h(store->parents.data() + so, o.parents, nsel * 4);
        d2h(store->tokens.data() + so, o.tokens, nsel * 4);
        d2h(store->lengths.data() + so, o.lengths, nsel * 4);
        d2h(store->raw.data() + so, o.raw_scores, nsel * 4);
        d2h(store->scores.data() + so, o.scores, nsel * 4);
        d2h(store->weights.data() + so, o.weights, nsel * 4);
        d2h(store->flp.data() + so, o.from_logprob, nsel);
        d2h(store->pool_parents.data() + po, o.pool_parents, npool * 4);
        d2h(store->pool_tokens.data() + po, o.pool_tokens, npool * 4);
        d2h(store->pool_lengths.data() + po, o.pool_lengths, npool * 4);
        d2h(store->pool_raw.data() + po, o.pool_raw_scores, npool * 4);
        d2h(store->pool_scores.data() + po, o.pool_scores, npool * 4);
        d2h(store->relaxed.data() + po, o.relaxed_weights, npool * 4);
        d2h(store->pool_flp.data() + po, o.pool_from_logprob, npool);
        d2h(store->final_raw.data() + fo, o.final_raw_scores, nfin * 4);
        d2h(store->final_scores.data() + fo, o.final_scores, nfin * 4);
        dbs_host::check_cuda(cudaStreamSynchronize(s), "decode");
    }
    (void)h;
    (void)stats_handle;
    return store;
}

// Surrogate backward of one result on the device: uploads the example's
// trace, runs the reverse sweep and reads the gradient back.
std::unique_ptr<DBSBackwardHandle> run_backward(DBSDecoderHandle* h, const DBSResultHandle* r,
                                                const float* gsel, const float* grel, const float* gfin,
                                                bool sparse) {
    const ResultStore& st = *r->store;
    const ExampleInfo& e = r->info();
    const Options& opt = st.opt;
    if (e.K != h->options.beam_size) throw std::invalid_argument("forward result beam_size does not match decoder");
    if (e.P < e.K) throw std::invalid_argument("invalid relaxed pool size");
    const size_t sel = checked_mul(static_cast<size_t>(e.T), static_cast<size_t>(e.K), "selected gradient size overflow");
    const size_t dense_count = checked_mul(sel, static_cast<size_t>(e.V), "dense gradient size overflow");
    if (!sparse && opt.max_dense_gradient_elements >= 0 &&
        dense_count > static_cast<size_t>(h->options.max_dense_gradient_elements)) {
        throw std::length_error("dense gradient allocation exceeds max_dense_gradient_elements; use sparse backward");
    }
    auto out = std::make_unique<DBSBackwardHandle>();
    out->sparse = sparse;
    const size_t pool = static_cast<size_t>(e.T) * e.P;
    const size_t nsp = static_cast<size_t>(e.T) * (e.K + e.P);
    // inputs packed at their device offsets in pinned memory, one copy up;
    // results read back through the same buffer
    const size_t in_bytes = sel * (4 * 3 + 1 + 4 + 4) + pool * (4 * 4 + 1 + 4) + e.K * 8 + 32 * 16;
    ThreadStaging& ts = thread_staging(std::max(in_bytes, nsp * 12 + 64));
    cudaStream_t s = ts.s;
    DeviceBuffer tb(in_bytes, s);
    char* base = tb.as<char>();
    char* cur = base;
    auto take = [&](size_t n) {
        char* p = cur;
        cur += (n + 15) & ~static_cast<size_t>(15);
        return p;
    };
    auto h2d = [&](void* dst, const void* src, size_t n) {
        if (n) std::memcpy(ts.pinned + (static_cast<char*>(dst) - base), src, n);
    };
    dbs_host::BackwardInputs in;
    auto* d_par = reinterpret_cast<int32_t*>(take(sel * 4));
    auto* d_tok = reinterpret_cast<int32_t*>(take(sel * 4));
    auto* d_len = reinterpret_cast<int32_t*>(take(sel * 4));
    auto* d_flp = reinterpret_cast<uint8_t*>(take(sel));
    h2d(d_par, st.parents.data() + e.sel, sel * 4);
    h2d(d_tok, st.tokens.data() + e.sel, sel * 4);
    h2d(d_len, st.lengths.data() + e.sel, sel * 4);
    h2d(d_flp, st.flp.data() + e.sel, sel);
    in.parents = d_par;
    in.tokens = d_tok;
    in.lengths = d_len;
    in.from_logprob = d_flp;
    if (gsel) {
        auto* d_w = reinterpret_cast<float*>(take(sel * 4));
        auto* d_g = reinterpret_cast<float*>(take(sel * 4));
        h2d(d_w, st.weights.data() + e.sel, sel * 4);
        h2d(d_g, gsel, sel * 4);
        in.weights = d_w;
        in.grad_selected = d_g;
    }
    if (grel) {
        auto* d_pp = reinterpret_cast<int32_t*>(take(pool * 4));
        auto* d_pt = reinterpret_cast<int32_t*>(take(pool * 4));
        auto* d_pl = reinterpret_cast<int32_t*>(take(pool * 4));
        auto* d_pf = reinterpret_cast<uint8_t*>(take(pool));
        auto* d_rw = reinterpret_cast<float*>(take(pool * 4));
        auto* d_rg = reinterpret_cast<float*>(take(pool * 4));
        h2d(d_pp, st.pool_parents.data() + e.pool, pool * 4);
        h2d(d_pt, st.pool_tokens.data() + e.pool, pool * 4);
        h2d(d_pl, st.pool_lengths.data() + e.pool, pool * 4);
        h2d(d_pf, st.pool_flp.data() + e.pool, pool);
        h2d(d_rw, st.relaxed.data() + e.pool, pool * 4);
        h2d(d_rg, grel, pool * 4);
        in.pool_parents = d_pp;
        in.pool_tokens = d_pt;
        in.pool_lengths = d_pl;
        in.pool_from_logprob = d_pf;
        in.relaxed_weights = d_rw;
        in.grad_relaxed = d_rg;
    }
    if (gfin) {
        auto* d_gf = reinterpret_cast<float*>(take(static_cast<size_t>(e.K) * 4));
        h2d(d_gf, gfin, static_cast<size_t>(e.K) * 4);
        in.grad_final = d_gf;
    }
    auto* d_gi = reinterpret_cast<float*>(take(static_cast<size_t>(e.K) * 4));
    const size_t staged = static_cast<size_t>(reinterpret_cast<char*>(d_gi) - base);
    dbs_host::check_cuda(cudaMemcpyAsync(base, ts.pinned, staged, cudaMemcpyHostToDevice, s), "stage trace");
    std::vector<ExampleSpec> spec(1);
    spec[0].T = e.T;
    spec[0].K = e.K;
    Options bopt = opt;
    const Layout L = dbs_host::make_layout(bopt, spec, e.V);
    dbs_host::BackwardOutputs bo;
    bo.grad_initial = d_gi;
    std::unique_ptr<DeviceBuffer> gbuf;
    int64_t nnz = 0;
    if (sparse) {
        gbuf.reset(new DeviceBuffer(nsp * (8 + 4) + 64, s));
        bo.sparse_indices = gbuf->as<int64_t>();
        bo.sparse_values = reinterpret_cast<float*>(bo.sparse_indices + nsp);
        bo.sparse_counts = reinterpret_cast<int64_t*>(take(8));
    } else {
        gbuf.reset(new DeviceBuffer(dense_count * 4, s));
        bo.grad_dense = gbuf->as<float>();
    }
    dbs_host::backward(bopt, e.V, spec, L, in, bo, s, true);
    host_alloc(out->grad_initial, static_cast<size_t>(e.K), 0.0f);
    // grad_initial and the count (adjacent on the device) in one copy
    const size_t gi_bytes = static_cast<size_t>(reinterpret_cast<char*>(sparse ? reinterpret_cast<char*>(bo.sparse_counts) + 8
                                                                                : reinterpret_cast<char*>(d_gi) + e.K * 4) -
                                                reinterpret_cast<char*>(d_gi));
    dbs_host::check_cuda(cudaMemcpyAsync(ts.pinned, d_gi, gi_bytes, cudaMemcpyDeviceToHost, s), "read grad_initial");
    dbs_host::check_cuda(cudaStreamSynchronize(s), "backward");
    std::memcpy(out->grad_initial.data(), ts.pinned, static_cast<size_t>(e.K) * 4);
    if (sparse) {
        std::memcpy(&nnz, ts.pinned + (reinterpret_cast<char*>(bo.sparse_counts) - reinterpret_cast<char*>(d_gi)), 8);
        host_alloc(out->indices, static_cast<size_t>(nnz), int64_t{0});
        host_alloc(out->values, static_cast<size_t>(nnz), 0.0f);
        if (nnz) {
            // indices and values are adjacent on the device: one copy
            dbs_host::check_cuda(cudaMemcpyAsync(ts.pinned, bo.sparse_indices, nsp * 8 + nnz * 4,
                                                 cudaMemcpyDeviceToHost, s),
                                 "read sparse entries");
            dbs_host::check_cuda(cudaStreamSynchronize(s), "backward");
            std::memcpy(out->indices.data(), ts.pinned, static_cast<size_t>(nnz) * 8);
            std::memcpy(out->values.data(), ts.pinned + nsp * 8, static_cast<size_t>(nnz) * 4);
        }
    } else {
        host_alloc(out->grad_log_probs, dense_count, 0.0f);
        dbs_host::check_cuda(cudaMemcpyAsync(out->grad_log_probs.data(), bo.grad_dense, dense_count * 4,
                                             cudaMemcpyDeviceToHost, s),
                             "read dense gradient");
    }
    dbs_host::check_cuda(cudaStreamSynchronize(s), "backward");
    return out;
}

template <class F>
int guarded(DBSDecoderHandle* h, F&& body) {
    try {
        return body();
    } catch (const std::exception& e) {
        set_error(h, e.what());
        mark_error(h, classify(e));
        return -2;
    } catch (...) {
        set_error(h, "unknown exception");
        mark_error(h, 2);
        return -3;
    }
}


}  // namespace

// ---------------------------------------------------------------------------
// Exported C ABI
// ---------------------------------------------------------------------------
extern "C" {

DBS_EXPORT int dbs_abi_version(void) { return DBS_ABI_VERSION; }
DBS_EXPORT const char* dbs_version_string(void) { return "1.0.0"; }
DBS_EXPORT const char* dbs_last_global_error(void) { return g_last_error.c_str(); }

DBS_EXPORT int dbs_workspace_create(DBSWorkspaceHandle** out_workspace) {
    if (out_workspace) *out_workspace = nullptr;
    if (!out_workspace) {
        set_error(nullptr, "out_workspace cannot be null");
        return -1;
    }
    try {
        *out_workspace = new DBSWorkspaceHandle;
        return 0;
    } catch (const std::exception& e) {
        set_error(nullptr, e.what());
        return -2;
    }
}

DBS_EXPORT void dbs_workspace_destroy(DBSWorkspaceHandle* workspace) { delete workspace; }

DBS_EXPORT int dbs_workspace_reserve(DBSWorkspaceHandle* workspace, int64_t float_count, int64_t int_count) {
    if (!workspace || float_count < 0 || int_count < 0) return -1;
    try {
        std::lock_guard<std::mutex> lock(workspace->mutex);
        workspace->f32.reserve(static_cast<size_t>(float_count));
        workspace->i32.reserve(static_cast<size_t>(int_count));
        return 0;
    } catch (...) {
        return -2;
    }
}

DBS_EXPORT int64_t dbs_workspace_allocated_bytes(DBSWorkspaceHandle* workspace) {
    if (!workspace) return 0;
    std::lock_guard<std::mutex> lock(workspace->mutex);
    return static_cast<int64_t>(workspace->f32.capacity() * sizeof(float) +
                                workspace->i32.capacity() * sizeof(int32_t));
}

DBS_EXPORT int dbs_create_ex(DBSOptionsC options, DBSDecoderHandle** out_handle) {
    if (out_handle) *out_handle = nullptr;
    if (!out_handle) {
        set_error(nullptr, "out_handle cannot be null");
        return -1;
    }
    try {
        auto h = std::make_unique<DBSDecoderHandle>();
        Options o = parse_options(options);
        check_options(o);
        h->options = o;
        h->beam_size = o.beam_size;
        h->stats.abi_version = DBS_ABI_VERSION;
        h->stats.last_kernel = kKernelCuda;
        DBSDecoderHandle* raw = h.get();
        *out_handle = h.release();
        clear_error(raw);
        return 0;
    } catch (const std::exception& e) {
        set_error(nullptr, e.what());
        return -2;
    } catch (...) {
        set_error(nullptr, "unknown exception");
        return -3;
    }
}

DBS_EXPORT DBSDecoderHandle* dbs_create(DBSOptionsC options) {
    DBSDecoderHandle* h = nullptr;
    return dbs_create_ex(options, &h) == 0 ? h : nullptr;
}

DBS_EXPORT void dbs_destroy(DBSDecoderHandle* handle) { delete handle; }

DBS_EXPORT const char* dbs_last_error(DBSDecoderHandle* handle) {
    if (!handle) return dbs_last_global_error();
    std::lock_guard<std::mutex> lock(handle->error_mutex);
    return handle->last_error.c_str();
}

static int decode_constrained_impl(DBSDecoderHandle* handle, const float* log_probs, int steps, int vocab_size,
                                   const uint8_t* banned, const int32_t* forced, int min_length, float rep,
                                   int ngram, const DBSAdvancedConstraintsC* filter_src,
                                   DBSResultHandle** out_result) {
    const int64_t t0 = now_ns();
    const Options& opt = handle->options;
    std::vector<int32_t> forced_host;
    if (forced && steps > 0) forced_host = host_copy(forced, static_cast<size_t>(steps));
    check_example(opt, log_probs, steps, vocab_size, opt.beam_size, opt.eos_token,
                  forced ? forced_host.data() : nullptr);
    HostExample e;
    e.T = steps;
    e.K = opt.beam_size;
    e.k_stride = opt.beam_size;
    e.eos = opt.eos_token;
    e.min_length = min_length >= 0 ? min_length : opt.min_length;
    e.banned = banned;
    e.forced = forced;
    CallConstraints cons;
    cons.repetition_penalty = rep;
    cons.no_repeat_ngram = ngram;
    dbs_host::TokenFilter filter;
    if (filter_src && filter_src->token_filter) {
        // the reference calls the filter with the constraints' batch index,
        // the step, the parent beam, its token prefix and the token
        const DBSTokenFilterFn fn = filter_src->token_filter;
        void* user = filter_src->token_filter_user_data;
        const int batch_index = filter_src->batch_index;
        filter = [fn, user, batch_index](int step, int parent, const int32_t* prefix, int prefix_len, int token) {
            return fn(user, batch_index, step, parent, prefix, prefix_len, token);
        };
    }
    auto store = run_decode(handle, opt, log_probs, vocab_size, {e}, cons, handle, filter ? &filter : nullptr);
    auto r = std::make_unique<DBSResultHandle>();
    r->store = store;
    r->index = 0;
    record_decode(handle, store->ex[0], now_ns() - t0, 1, false);
    *out_result = r.release();
    clear_error(handle);
    return 0;
}

DBS_EXPORT int dbs_decode(DBSDecoderHandle* handle, const float* log_probs, int steps, int vocab_size,
                          DBSResultHandle** out_result) {
    if (out_result) *out_result = nullptr;
    if (!handle || !out_result) return -1;
    return guarded(handle, [&]() {
        return decode_constrained_impl(handle, log_probs, steps, vocab_size, nullptr, nullptr, -1, 1.0f, 0, nullptr,
                                       out_result);
    });
}

DBS_EXPORT int dbs_decode_constrained(DBSDecoderHandle* handle, const float* log_probs, int steps, int vocab_size,
                                      const uint8_t* banned_tokens, const int32_t* forced_tokens, int min_length,
                                      DBSResultHandle** out_result) {
    DBSAdvancedConstraintsC c{};
    c.banned_tokens = banned_tokens;
    c.forced_tokens = forced_tokens;
    c.min_length = min_length;
    c.repetition_penalty = 1.0f;
    c.no_repeat_ngram_size = 0;
    return dbs_decode_constrained_ex(handle, log_probs, steps, vocab_size, &c, out_result);
}

DBS_EXPORT int dbs_decode_constrained_ex(DBSDecoderHandle* handle, const float* log_probs, int steps,
                                         int vocab_size, const DBSAdvancedConstraintsC* c,
                                         DBSResultHandle** out_result) {
    if (out_result) *out_result = nullptr;
    if (!handle || !out_result) {
        set_error(handle, "invalid decoder, result, or output pointer");
        mark_error(handle, 1);
        return -1;
    }
    return guarded(handle, [&]() {
        const uint8_t* banned = c ? c->banned_tokens : nullptr;
        const int32_t* forced = c ? c->forced_tokens : nullptr;
        const int min_length = c ? c->min_length : -1;
        const float rep = (c && c->repetition_penalty > 0.0f) ? c->repetition_penalty : 1.0f;
        const int ngram = c ? c->no_repeat_ngram_size : 0;
        return decode_constrained_impl(handle, log_probs, steps, vocab_size, banned, forced, min_length, rep, ngram,
                                       c, out_result);
    });
}

DBS_EXPORT int dbs_decode_batch(DBSDecoderHandle* handle, const float* log_probs, int batch_size, int steps,
                                int vocab_size, int num_threads, DBSBatchResultHandle** out_result) {
    if (out_result) *out_result = nullptr;
    if (!handle || !out_result) {
        set_error(handle, "invalid decoder, result, or output pointer");
        return -1;
    }
    if (!log_probs || batch_size <= 0 || steps <= 0 || vocab_size <= 0) {
        set_error(handle, "invalid batch decode arguments");
        return -1;
    }
    (void)num_threads;
    return guarded(handle, [&]() {
        const int64_t t0 = now_ns();
        const Options& opt = handle->options;
        const size_t step_beam = checked_mul(static_cast<size_t>(steps), static_cast<size_t>(opt.beam_size),
                                             "batch stride overflow");
        const size_t stride = checked_mul(step_beam, static_cast<size_t>(vocab_size), "batch stride overflow");
        std::vector<HostExample> hx(static_cast<size_t>(batch_size));
        for (int b = 0; b < batch_size; ++b) {
            check_example(opt, log_probs, steps, vocab_size, opt.beam_size, opt.eos_token, nullptr);
            hx[b].T = steps;
            hx[b].K = opt.beam_size;
            hx[b].k_stride = opt.beam_size;
            hx[b].eos = opt.eos_token;
            hx[b].min_length = opt.min_length;
            hx[b].x_offset = static_cast<int64_t>(stride) * b;
        }
        auto store = run_decode(handle, opt, log_probs, vocab_size, hx, CallConstraints{}, handle);
        auto br = std::make_unique<DBSBatchResultHandle>();
        br->store = store;
        br->items.resize(static_cast<size_t>(batch_size));
        for (int b = 0; b < batch_size; ++b) {
            br->items[b].store = store;
            br->items[b].index = b;
        }
        record_decode(handle, store->ex[0], now_ns() - t0, 1, false);
        *out_result = br.release();
        clear_error(handle);
        return 0;
    });
}

DBS_EXPORT int dbs_decode_batch_variable(DBSDecoderHandle* handle, const float* log_probs, int batch_size,
                                         int max_steps, int max_beam_size, int vocab_size,
                                         const int32_t* steps_per_example, const int32_t* beam_sizes_per_example,
                                         const int32_t* eos_tokens_per_example,
                                         const int32_t* min_lengths_per_example,
                                         const uint8_t* banned_tokens_per_example,
                                         const int32_t* forced_tokens_per_example, int num_threads,
                                         DBSBatchResultHandle** out_result) {
    if (out_result) *out_result = nullptr;
    if (!handle || !log_probs || !out_result || batch_size <= 0 || max_steps <= 0 || max_beam_size <= 0 ||
        vocab_size <= 0) {
        set_error(handle, "invalid variable batch decode arguments");
        mark_error(handle, 1);
        return -1;
    }
    (void)num_threads;
    return guarded(handle, [&]() {
        const int64_t t0 = now_ns();
        const size_t B = static_cast<size_t>(batch_size);
        const std::vector<int32_t> steps_h = host_copy(steps_per_example, steps_per_example ? B : 0);
        const std::vector<int32_t> beams_h = host_copy(beam_sizes_per_example, beam_sizes_per_example ? B : 0);
        const std::vector<int32_t> eos_h = host_copy(eos_tokens_per_example, eos_tokens_per_example ? B : 0);
        const std::vector<int32_t> minlen_h = host_copy(min_lengths_per_example, min_lengths_per_example ? B : 0);
        const std::vector<int32_t> forced_h = host_copy(
            forced_tokens_per_example, forced_tokens_per_example ? B * static_cast<size_t>(max_steps) : 0);
        const size_t input_stride =
            static_cast<size_t>(max_steps) * static_cast<size_t>(max_beam_size) * static_cast<size_t>(vocab_size);
        std::vector<HostExample> hx(B);
        for (size_t b = 0; b < B; ++b) {
            // dbs_decode_batch_variable worker, src/differentiable_beam.cpp:3722-3751
            const int steps = steps_per_example ? steps_h[b] : max_steps;
            const int beam = beam_sizes_per_example ? beams_h[b] : handle->beam_size;
            if (steps <= 0 || steps > max_steps) throw std::invalid_argument("invalid per-example steps");
            if (beam <= 0 || beam > max_beam_size) throw std::invalid_argument("invalid per-example beam size");
            Options eopt = handle->options;
            eopt.beam_size = beam;
            if (eos_tokens_per_example) eopt.eos_token = eos_h[b];
            if (min_lengths_per_example) eopt.min_length = std::max(0, minlen_h[b]);
            check_options(eopt);
            const int32_t* fh = forced_tokens_per_example ? forced_h.data() + b * max_steps : nullptr;
            check_example(eopt, log_probs, steps, vocab_size, beam, eopt.eos_token, fh);
            const int cmin = min_lengths_per_example ? minlen_h[b] : -1;
            hx[b].T = steps;
            hx[b].K = beam;
            hx[b].k_stride = max_beam_size;
            hx[b].eos = eopt.eos_token;
            hx[b].min_length = cmin >= 0 ? cmin : eopt.min_length;
            hx[b].x_offset = static_cast<int64_t>(input_stride * b);
            hx[b].banned = banned_tokens_per_example ? banned_tokens_per_example + b * static_cast<size_t>(vocab_size)
                                                     : nullptr;
            hx[b].forced = forced_tokens_per_example ? forced_tokens_per_example + b * static_cast<size_t>(max_steps)
                                                     : nullptr;
        }
        auto store = run_decode(handle, handle->options, log_probs, vocab_size, hx, CallConstraints{}, handle);
        auto br = std::make_unique<DBSBatchResultHandle>();
        br->store = store;
        br->items.resize(B);
        for (size_t b = 0; b < B; ++b) {
            br->items[b].store = store;
            br->items[b].index = static_cast<int>(b);
        }
        record_decode(handle, store->ex[0], now_ns() - t0, 1, false);
        *out_result = br.release();
        clear_error(handle);
        return 0;
    });
}

// fp16 / bf16 inputs are widened to fp32 on the device (exact), then decoded.
static int decode_typed_impl(DBSDecoderHandle* handle, const void* log_probs, int data_type, int batch, int steps,
                             int vocab_size, bool batched, DBSResultHandle** out_r, DBSBatchResultHandle** out_b) {
    const int64_t count = static_cast<int64_t>(batched ? batch : 1) * steps * handle->beam_size * vocab_size;
    if (count <= 0) {
        throw std::invalid_argument(batched ? "typed batch decode dimensions must be positive"
                                            : "typed decode dimensions must be positive");
    }
    if (data_type == DBS_DTYPE_F32) {
        return batched ? dbs_decode_batch(handle, static_cast<const float*>(log_probs), batch, steps, vocab_size, 0,
                                          out_b)
                       : dbs_decode(handle, static_cast<const float*>(log_probs), steps, vocab_size, out_r);
    }
    if (!log_probs) throw std::invalid_argument("typed log_probs cannot be null");
    if (data_type != DBS_DTYPE_F16 && data_type != DBS_DTYPE_BF16)
        throw std::invalid_argument("unsupported DBS data type");
    CallStream cs(nullptr);
    DeviceBuffer src(is_device_pointer(log_probs) ? 0 : static_cast<size_t>(count) * 2, cs.s);
    const uint16_t* d_src = static_cast<const uint16_t*>(log_probs);
    if (src.ptr) {
        dbs_host::check_cuda(cudaMemcpyAsync(src.ptr, log_probs, static_cast<size_t>(count) * 2,
                                             cudaMemcpyHostToDevice, cs.s),
                             "stage typed log_probs");
        d_src = src.as<uint16_t>();
    }
    dbs_host::check_cuda(cudaStreamSynchronize(cs.s), "stage typed log_probs");
    // the decode reads the 16-bit values natively (exact widening on load)
    const int64_t t0 = now_ns();
    const Options& opt = handle->options;
    const int B = batched ? batch : 1;
    const int64_t stride = static_cast<int64_t>(steps) * opt.beam_size * vocab_size;
    std::vector<HostExample> hx(static_cast<size_t>(B));
    for (int b = 0; b < B; ++b) {
        check_example(opt, reinterpret_cast<const float*>(d_src), steps, vocab_size, opt.beam_size, opt.eos_token,
                      nullptr);
        hx[b].T = steps;
        hx[b].K = opt.beam_size;
        hx[b].k_stride = opt.beam_size;
        hx[b].eos = opt.eos_token;
        hx[b].min_length = opt.min_length;
        hx[b].x_offset = stride * b;
    }
    auto store = run_decode(handle, opt, nullptr, vocab_size, hx, CallConstraints{}, handle, nullptr, d_src,
                            data_type == DBS_DTYPE_BF16);
    if (batched) {
        auto br = std::make_unique<DBSBatchResultHandle>();
        br->store = store;
        br->items.resize(static_cast<size_t>(B));
        for (int b = 0; b < B; ++b) {
            br->items[b].store = store;
            br->items[b].index = b;
        }
        record_decode(handle, store->ex[0], now_ns() - t0, 1, false);
        *out_b = br.release();
    } else {
        auto r = std::make_unique<DBSResultHandle>();
        r->store = store;
        r->index = 0;
        record_decode(handle, store->ex[0], now_ns() - t0, 1, false);
        *out_r = r.release();
    }
    clear_error(handle);
    return 0;
}

DBS_EXPORT int dbs_decode_typed(DBSDecoderHandle* handle, const void* log_probs, int data_type, int steps,
                                int vocab_size, DBSResultHandle** out_result) {
    if (out_result) *out_result = nullptr;
    if (!handle || !out_result) return -1;
    return guarded(handle, [&]() {
        return decode_typed_impl(handle, log_probs, data_type, 1, steps, vocab_size, false, out_result, nullptr);
    });
}

DBS_EXPORT int dbs_decode_batch_typed(DBSDecoderHandle* handle, const void* log_probs, int data_type,
                                      int batch_size, int steps, int vocab_size, int num_threads,
                                      DBSBatchResultHandle** out_result) {
    if (out_result) *out_result = nullptr;
    if (!handle || !out_result) return -1;
    (void)num_threads;
    return guarded(handle, [&]() {
        return decode_typed_impl(handle, log_probs, data_type, batch_size, steps, vocab_size, true, nullptr,
                                 out_result);
    });
}

DBS_EXPORT int dbs_decode_model_steps(DBSDecoderHandle* handle, DBSModelStepFn step_fn, void* user_data,
                                      int batch_index, int steps, int vocab_size, DBSResultHandle** out_result) {
    DBSWorkspaceHandle local;
    return dbs_decode_model_steps_with_workspace(handle, &local, step_fn, user_data, batch_index, steps, vocab_size,
                                                 out_result);
}

// The model-step decode of src/differentiable_beam.cpp:3506-3586: the callback
// fills step t's [K,V] rows from the previous step's tokens and final scores,
// which come from a device decode of the first t+1 steps.
DBS_EXPORT int dbs_decode_model_steps_with_workspace(DBSDecoderHandle* handle, DBSWorkspaceHandle* workspace,
                                                     DBSModelStepFn step_fn, void* user_data, int batch_index,
                                                     int steps, int vocab_size, DBSResultHandle** out_result) {
    if (out_result) *out_result = nullptr;
    if (!handle || !workspace || !step_fn || !out_result) {
        set_error(handle, "invalid decoder, workspace, model step callback, or output pointer");
        mark_error(handle, 1);
        return -1;
    }
    if (steps <= 0 || vocab_size <= 0) {
        set_error(handle, "steps and vocab_size must be positive");
        mark_error(handle, 1);
        return -1;
    }
    return guarded(handle, [&]() {
        const int64_t t0 = now_ns();
        const int K = handle->beam_size;
        const size_t row_count = static_cast<size_t>(K) * static_cast<size_t>(vocab_size);
        const size_t total = static_cast<size_t>(steps) * row_count;
        std::lock_guard<std::mutex> lock(workspace->mutex);
        workspace->f32.assign(total, -std::numeric_limits<float>::infinity());
        workspace->i32.assign(static_cast<size_t>(K), -1);
        std::vector<float> prev_scores_buf(static_cast<size_t>(K), 0.0f);
        const Options& opt = handle->options;
        // The callback fills step t's rows from the previous step's tokens
        // and the final scores of the decode so far; the device decodes one
        // step per launch and keeps the beams between launches, so the work
        // grows linearly with the steps (the reference re-decodes every
        // prefix).
        dbs_host::StepRows rows = [&](int t, const int32_t* prev_tokens, const float* prev_scores, float* d_rows) {
            float* row = workspace->f32.data() + static_cast<size_t>(t) * row_count;
            for (int k = 0; k < K; ++k) {
                workspace->i32[static_cast<size_t>(k)] = prev_tokens[k];
                prev_scores_buf[static_cast<size_t>(k)] = prev_scores[k];
            }
            const int rc = step_fn(user_data, batch_index, t, workspace->i32.data(), prev_scores_buf.data(), K,
                                   vocab_size, row);
            if (rc != 0) throw std::runtime_error("model step callback returned non-zero status");
            if (opt.validate_inputs) {
                // the reference validates every prefix it decodes (steps
                // 0..t), sampling 1000 evenly spaced elements of each
                // (validate_logprob_tensor, src/differentiable_beam.cpp:385-402)
                const size_t count = static_cast<size_t>(t + 1) * row_count;
                const size_t stride = count > 1000 ? count / 1000 : 1;
                for (size_t i = 0; i < count; i += stride) {
                    const float v = workspace->f32[i];
                    if (std::isnan(v) || v == std::numeric_limits<float>::infinity())
                        throw std::invalid_argument("log_probs contains NaN or +Inf");
                }
            }
            dbs_host::check_cuda(cudaMemcpy(d_rows, row, row_count * sizeof(float), cudaMemcpyHostToDevice),
                                 "upload model step rows");
        };
        HostExample e;
        e.T = steps;
        e.K = K;
        e.k_stride = K;
        e.eos = opt.eos_token;
        e.min_length = opt.min_length;
        auto store = run_decode(handle, opt, nullptr, vocab_size, {e}, CallConstraints{}, handle, nullptr, nullptr,
                                false, &rows);
        auto r = std::make_unique<DBSResultHandle>();
        r->store = store;
        record_decode(handle, store->ex[0], now_ns() - t0, 1, true);
        {
            const int64_t ws_bytes = static_cast<int64_t>(workspace->f32.capacity() * sizeof(float) +
                                                          workspace->i32.capacity() * sizeof(int32_t));
            std::lock_guard<std::mutex> slock(handle->stats_mutex);
            handle->stats.last_allocation_bytes += ws_bytes;
        }
        *out_result = r.release();
        clear_error(handle);
        return 0;
    });
}

static int backward_entry(DBSDecoderHandle* handle, const DBSResultHandle* result, const float* gsel,
                          const float* grel, const float* gfin, DBSBackwardHandle** out, bool sparse) {
    if (out) *out = nullptr;
    if (!handle || !result || !out) {
        set_error(handle, "invalid decoder, result, or output pointer");
        mark_error(handle, 1);
        return -1;
    }
    return guarded(handle, [&]() {
        const int64_t t0 = now_ns();
        auto b = run_backward(handle, result, gsel, grel, gfin, sparse);
        record_backward(handle, *b, now_ns() - t0);
        *out = b.release();
        clear_error(handle);
        return 0;
    });
}

DBS_EXPORT int dbs_backward(DBSDecoderHandle* handle, const DBSResultHandle* result, const float* gsel,
                            const float* grel, const float* gfin, DBSBackwardHandle** out_backward) {
    return backward_entry(handle, result, gsel, grel, gfin, out_backward, true);
}
DBS_EXPORT int dbs_backward_sparse(DBSDecoderHandle* handle, const DBSResultHandle* result, const float* gsel,
                                   const float* grel, const float* gfin, DBSBackwardHandle** out_backward) {
    return backward_entry(handle, result, gsel, grel, gfin, out_backward, true);
}
DBS_EXPORT int dbs_backward_default(DBSDecoderHandle* handle, const DBSResultHandle* result, const float* gsel,
                                    const float* grel, const float* gfin, DBSBackwardHandle** out_backward) {
    return backward_entry(handle, result, gsel, grel, gfin, out_backward, true);
}
DBS_EXPORT int dbs_backward_dense(DBSDecoderHandle* handle, const DBSResultHandle* result, const float* gsel,
                                  const float* grel, const float* gfin, DBSBackwardHandle** out_backward) {
    return backward_entry(handle, result, gsel, grel, gfin, out_backward, false);
}

DBS_EXPORT void dbs_free_result(DBSResultHandle* result) { delete result; }
DBS_EXPORT void dbs_free_batch_result(DBSBatchResultHandle* result) { delete result; }
DBS_EXPORT void dbs_free_backward(DBSBackwardHandle* result) { delete result; }

DBS_EXPORT int dbs_batch_result_size(const DBSBatchResultHandle* result) {
    return result ? static_cast<int>(result->items.size()) : 0;
}
DBS_EXPORT const DBSResultHandle* dbs_batch_result_at(const DBSBatchResultHandle* result, int batch_index) {
    if (!result || batch_index < 0 || batch_index >= static_cast<int>(result->items.size())) return nullptr;
    return &result->items[static_cast<size_t>(batch_index)];
}

DBS_EXPORT int dbs_result_steps(const DBSResultHandle* r) { return r ? r->info().T : 0; }
DBS_EXPORT int dbs_result_beam_size(const DBSResultHandle* r) { return r ? r->info().K : 0; }
DBS_EXPORT int dbs_result_vocab_size(const DBSResultHandle* r) { return r ? r->info().V : 0; }
DBS_EXPORT int dbs_result_pool_size(const DBSResultHandle* r) { return r ? r->info().P : 0; }

#define DBS_SEL_ACCESSOR(name, type, field) \
    DBS_EXPORT const type* name(const DBSResultHandle* r) { return r ? r->store->field.data() + r->info().sel : nullptr; }
#define DBS_POOL_ACCESSOR(name, type, field) \
    DBS_EXPORT const type* name(const DBSResultHandle* r) { return r ? r->store->field.data() + r->info().pool : nullptr; }
#define DBS_FINAL_ACCESSOR(name, type, field) \
    DBS_EXPORT const type* name(const DBSResultHandle* r) { return r ? r->store->field.data() + r->info().fin : nullptr; }

DBS_SEL_ACCESSOR(dbs_result_tokens, int32_t, tokens)
DBS_SEL_ACCESSOR(dbs_result_parents, int32_t, parents)
DBS_SEL_ACCESSOR(dbs_result_lengths, int32_t, lengths)
DBS_SEL_ACCESSOR(dbs_result_scores, float, scores)
DBS_SEL_ACCESSOR(dbs_result_raw_scores, float, raw)
DBS_SEL_ACCESSOR(dbs_result_weights, float, weights)
DBS_FINAL_ACCESSOR(dbs_result_final_scores, float, final_scores)
DBS_FINAL_ACCESSOR(dbs_result_final_raw_scores, float, final_raw)
DBS_POOL_ACCESSOR(dbs_result_relaxed_weights, float, relaxed)
DBS_POOL_ACCESSOR(dbs_result_pool_tokens, int32_t, pool_tokens)
DBS_POOL_ACCESSOR(dbs_result_pool_parents, int32_t, pool_parents)
DBS_POOL_ACCESSOR(dbs_result_pool_lengths, int32_t, pool_lengths)
DBS_POOL_ACCESSOR(dbs_result_pool_scores, float, pool_scores)
DBS_POOL_ACCESSOR(dbs_result_pool_raw_scores, float, pool_raw)

DBS_EXPORT const float* dbs_backward_grad_log_probs(const DBSBackwardHandle* b) {
    return b ? b->grad_log_probs.data() : nullptr;
}
DBS_EXPORT const float* dbs_backward_grad_initial_scores(const DBSBackwardHandle* b) {
    return b ? b->grad_initial.data() : nullptr;
}
DBS_EXPORT const int64_t* dbs_backward_sparse_logprob_indices(const DBSBackwardHandle* b) {
    return b ? b->indices.data() : nullptr;
}
DBS_EXPORT const float* dbs_backward_sparse_logprob_values(const DBSBackwardHandle* b) {
    return b ? b->values.data() : nullptr;
}
DBS_EXPORT int64_t dbs_backward_sparse_logprob_count(const DBSBackwardHandle* b) {
    return b ? static_cast<int64_t>(b->values.size()) : 0;
}
DBS_EXPORT int dbs_backward_is_sparse(const DBSBackwardHandle* b) { return b && b->sparse ? 1 : 0; }

DBS_EXPORT int64_t dbs_result_selected_count(const DBSResultHandle* r) {
    return r ? static_cast<int64_t>(r->info().T) * r->info().K : 0;
}
DBS_EXPORT int64_t dbs_result_pool_count(const DBSResultHandle* r) {
    return r ? static_cast<int64_t>(r->info().T) * r->info().P : 0;
}
DBS_EXPORT int64_t dbs_result_logprob_count(const DBSResultHandle* r) {
    return r ? static_cast<int64_t>(r->info().T) * r->info().K * r->info().V : 0;
}
DBS_EXPORT int64_t dbs_backward_grad_log_probs_count(const DBSResultHandle* r) { return dbs_result_logprob_count(r); }
DBS_EXPORT int64_t dbs_backward_grad_initial_scores_count(const DBSResultHandle* r) { return r ? r->info().K : 0; }

DBS_EXPORT int64_t dbs_result_eos_count(const DBSResultHandle* r, int eos_token) {
    if (!r || eos_token < 0) return 0;
    const int32_t* tok = dbs_result_tokens(r);
    const int64_t n = dbs_result_selected_count(r);
    int64_t c = 0;
    for (int64_t i = 0; i < n; ++i) c += tok[i] == eos_token;
    return c;
}

// Ordering check of src/differentiable_beam.cpp:4043-4065.
DBS_EXPORT int dbs_result_validate_deterministic_order(const DBSResultHandle* r) {
    if (!r) return -1;
    const int T = r->info().T, K = r->info().K;
    if (T < 0 || K < 0) return -2;
    const float* sc = dbs_result_scores(r);
    const int32_t* par = dbs_result_parents(r);
    const int32_t* tok = dbs_result_tokens(r);
    for (int t = 0; t < T; ++t) {
        for (int k = 1; k < K; ++k) {
            const size_t a = static_cast<size_t>(t) * K + (k - 1), b = a + 1;
            if (std::isfinite(sc[a]) && std::isfinite(sc[b]) && sc[b] > sc[a]) return -3;
            if (sc[a] == sc[b]) {
                if (par[b] < par[a] || (par[b] == par[a] && tok[b] < tok[a])) return -4;
            }
        }
    }
    return 0;
}

// Summary of src/differentiable_beam.cpp:4067-4102 (same keys and format).
DBS_EXPORT int dbs_result_summary_json(const DBSResultHandle* r, int eos_token, char* out_json, int64_t cap) {
    if (!r || !out_json || cap <= 0) return -1;
    const ExampleInfo& e = r->info();
    const int64_t n = static_cast<int64_t>(e.T) * e.K;
    const int32_t* len = dbs_result_lengths(r);
    int min_len = n ? std::numeric_limits<int>::max() : 0, max_len = 0;
    for (int64_t i = 0; i < n; ++i) {
        min_len = std::min(min_len, static_cast<int>(len[i]));
        max_len = std::max(max_len, static_cast<int>(len[i]));
    }
    const float* fs = dbs_result_final_scores(r);
    float mn = e.K ? fs[0] : 0.0f, mx = e.K ? fs[0] : 0.0f;
    for (int k = 0; k < e.K; ++k) {
        if (fs[k] < mn) mn = fs[k];
        if (fs[k] > mx) mx = fs[k];
    }
    const int w = std::snprintf(
        out_json, static_cast<size_t>(cap),
        "{\"abi_version\":%d,\"steps\":%d,\"beam_size\":%d,\"vocab_size\":%d,\"selected_count\":%lld,"
        "\"pool_count\":%lld,\"eos_token\":%d,\"eos_count\":%lld,\"min_length\":%d,\"max_length\":%d,"
        "\"min_final_score\":%.9g,\"max_final_score\":%.9g,\"deterministic_order\":%d}",
        DBS_ABI_VERSION, e.T, e.K, e.V, static_cast<long long>(n), static_cast<long long>(e.T) * e.P, eos_token,
        static_cast<long long>(dbs_result_eos_count(r, eos_token)), min_len, max_len, static_cast<double>(mn),
        static_cast<double>(mx), dbs_result_validate_deterministic_order(r) == 0 ? 1 : 0);
    if (w < 0) return -2;
    return w < cap ? 0 : 1;
}

DBS_EXPORT int dbs_validate_production_gate_manifest(const char* manifest_json, char* out_error, int64_t cap) {
    (void)manifest_json;
    if (out_error && cap > 0) {
        std::snprintf(out_error, static_cast<size_t>(cap), "%s",
                      "deprecated: release evidence cannot be validated by the C ABI; run tests and attach raw "
                      "benchmark/artifact logs");
    }
    return -1;
}

DBS_EXPORT int dbs_has_avx512(void) {
#if defined(__x86_64__)
    return __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("fma") ? 1 : 0;
#else
    return 0;
#endif
}
DBS_EXPORT int dbs_has_avx2(void) {
#if defined(__x86_64__)
    return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma") ? 1 : 0;
#else
    return 0;
#endif
}
DBS_EXPORT int dbs_has_sse42(void) {
#if defined(__x86_64__)
    return __builtin_cpu_supports("sse4.2") ? 1 : 0;
#else
    return 0;
#endif
}
DBS_EXPORT int dbs_has_neon(void) {
#if defined(__ARM_NEON) || defined(__ARM_NEON__)
    return 1;
#else
    return 0;
#endif
}
DBS_EXPORT const char* dbs_selected_kernel_name(void) { return "cuda"; }

DBS_EXPORT int dbs_get_stats(DBSDecoderHandle* handle, DBSStatsC* out_stats) {
    if (!handle || !out_stats) return -1;
    std::lock_guard<std::mutex> lock(handle->stats_mutex);
    *out_stats = handle->stats;
    out_stats->total_allocator_calls = g_alloc_calls.load(std::memory_order_relaxed);
    out_stats->total_allocator_bytes = g_alloc_bytes.load(std::memory_order_relaxed);
    return 0;
}

static const char* kernel_name(int k) {
    switch (k) {
        case 1: return "sse4.2";
        case 2: return "avx2";
        case 3: return "avx512";
        case 4: return "neon";
        case 5: return "cuda";
        default: return "scalar";
    }
}

DBS_EXPORT int dbs_get_stats_json(DBSDecoderHandle* handle, char* out_json, int64_t cap) {
    if (!handle || !out_json || cap <= 0) return -1;
    DBSStatsC s{};
    if (dbs_get_stats(handle, &s) != 0) return -1;
    const int w = std::snprintf(
        out_json, static_cast<size_t>(cap),
        "{\"abi_version\":%d,\"kernel\":\"%s\",\"used_sparse_backward\":%d,\"used_dense_backward\":%d,"
        "\"batch_threads\":%d,\"model_step\":%d,\"last_error_category\":%d,\"decode_ns\":%lld,\"backward_ns\":%lld,"
        "\"allocation_bytes\":%lld,\"selected_count\":%lld,\"pool_count\":%lld,\"logprob_count\":%lld,"
        "\"sparse_grad_count\":%lld,\"allocator_calls\":%lld,\"allocator_bytes\":%lld}",
        s.abi_version, kernel_name(s.last_kernel), s.used_sparse_backward, s.used_dense_backward, s.used_batch_threads,
        s.used_model_step_callback, s.last_error_category, static_cast<long long>(s.last_decode_ns),
        static_cast<long long>(s.last_backward_ns), static_cast<long long>(s.last_allocation_bytes),
        static_cast<long long>(s.last_selected_count), static_cast<long long>(s.last_pool_count),
        static_cast<long long>(s.last_logprob_count), static_cast<long long>(s.last_sparse_grad_count),
        static_cast<long long>(s.total_allocator_calls), static_cast<long long>(s.total_allocator_bytes));
    if (w < 0) return -2;
    return w < cap ? 0 : 1;
}

DBS_EXPORT int dbs_is_deterministic(void) { return 1; }

DBS_EXPORT int dbs_set_deterministic_seed(DBSDecoderHandle* handle, uint64_t seed) {
    if (!handle) return -1;
    handle->deterministic_seed = seed;
    return 0;
}
DBS_EXPORT uint64_t dbs_get_deterministic_seed(DBSDecoderHandle* handle) {
    return handle ? handle->deterministic_seed : 0;
}
DBS_EXPORT void dbs_allocator_counters_reset(void) {
    g_alloc_calls.store(0, std::memory_order_relaxed);
    g_alloc_bytes.store(0, std::memory_order_relaxed);
}
DBS_EXPORT int64_t dbs_allocator_call_count(void) { return g_alloc_calls.load(std::memory_order_relaxed); }
DBS_EXPORT int64_t dbs_allocator_byte_count(void) { return g_alloc_bytes.load(std::memory_order_relaxed); }
DBS_EXPORT void dbs_reset_stats(DBSDecoderHandle* handle) {
    if (!handle) return;
    std::lock_guard<std::mutex> lock(handle->stats_mutex);
    handle->stats = DBSStatsC{};
    handle->stats.abi_version = DBS_ABI_VERSION;
    handle->stats.last_kernel = kKernelCuda;
}

// ---------------------------------------------------------------------------
// Device-resident extension (include/dbs_device.h)
// ---------------------------------------------------------------------------
static dbs_host::Outputs to_outputs(const DBSDeviceDecodeOutputs* o) {
    dbs_host::Outputs r;
    r.parents = o->parents;
    r.tokens = o->tokens;
    r.lengths = o->lengths;
    r.from_logprob = o->from_logprob;
    r.raw_scores = o->raw_scores;
    r.scores = o->scores;
    r.weights = o->weights;
    r.pool_parents = o->pool_parents;
    r.pool_tokens = o->pool_tokens;
    r.pool_lengths = o->pool_lengths;
    r.pool_from_logprob = o->pool_from_logprob;
    r.pool_raw_scores = o->pool_raw_scores;
    r.pool_scores = o->pool_scores;
    r.relaxed_weights = o->relaxed_weights;
    r.final_raw_scores = o->final_raw_scores;
    r.final_scores = o->final_scores;
    return r;
}

static void run_device_decode(DBSDecoderHandle* handle, const float* x, int V, const std::vector<ExampleSpec>& spec,
                              const CallConstraints& cons, const DBSDeviceDecodeOutputs* outputs, void* stream,
                              float* zero_fill = nullptr, int64_t zero_fill_count = 0,
                              const dbs_host::DecodeControl* split = nullptr) {
    const Options& opt = handle->options;
    if (!outputs || !outputs->parents || !outputs->tokens || !outputs->lengths || !outputs->from_logprob)
        throw std::invalid_argument("device outputs need parents, tokens, lengths and from_logprob");
    const bool pool = outputs->pool_scores != nullptr;
    if (pool && (!outputs->pool_parents || !outputs->pool_tokens || !outputs->pool_lengths ||
                 !outputs->pool_raw_scores))
        throw std::invalid_argument("device pool outputs are incomplete");
    const Layout L = dbs_host::make_layout(opt, spec, V);
    dbs_host::DecodeStats st;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);  // NULL = legacy default stream
    dbs_host::DecodeControl ctl = split ? *split : dbs_host::DecodeControl{};
    ctl.synchronize = false;  // validation is still checked before the decode is queued
    ctl.zero_fill = zero_fill;
    ctl.zero_fill_count = zero_fill_count;
    dbs_host::decode(opt, x, V, spec, cons, to_outputs(outputs), L, pool, outputs->weights != nullptr, s, &st,
                     ctl);
    (void)handle;
}

DBS_EXPORT int dbs_device_decode_batch_ex(DBSDecoderHandle* handle, const float* log_probs, int batch_size,
                                          int steps, int vocab_size, const DBSDeviceDecodeOutputs* outputs,
                                          float* zero_fill, int64_t zero_fill_count, void* cuda_stream);

DBS_EXPORT int dbs_device_decode_batch(DBSDecoderHandle* handle, const float* log_probs, int batch_size, int steps,
                                       int vocab_size, const DBSDeviceDecodeOutputs* outputs, void* cuda_stream) {
    return dbs_device_decode_batch_ex(handle, log_probs, batch_size, steps, vocab_size, outputs, nullptr, 0,
                                      cuda_stream);
}

DBS_EXPORT int dbs_device_decode_batch_ex(DBSDecoderHandle* handle, const float* log_probs, int batch_size,
                                          int steps, int vocab_size, const DBSDeviceDecodeOutputs* outputs,
                                          float* zero_fill, int64_t zero_fill_count, void* cuda_stream) {
    if (!handle || !outputs) {
        set_error(handle, "invalid decoder or output pointer");
        return -1;
    }
    return guarded(handle, [&]() {
        const int64_t t0 = now_ns();
        const Options& opt = handle->options;
        if (batch_size <= 0) throw std::invalid_argument("batch_size must be positive");
        check_example(opt, log_probs, steps, vocab_size, opt.beam_size, opt.eos_token, nullptr);
        const int64_t stride = static_cast<int64_t>(steps) * opt.beam_size * vocab_size;
        std::vector<ExampleSpec> spec(static_cast<size_t>(batch_size));
        for (int b = 0; b < batch_size; ++b) {
            spec[b].T = steps;
            spec[b].K = opt.beam_size;
            spec[b].k_stride = opt.beam_size;
            spec[b].x_offset = stride * b;
            spec[b].eos = opt.eos_token;
            spec[b].min_length = opt.min_length;
        }
        if (zero_fill_count < 0 || (zero_fill_count > 0 && !zero_fill))
            throw std::invalid_argument("zero_fill needs a buffer for a positive element count");
        run_device_decode(handle, log_probs, vocab_size, spec, CallConstraints{}, outputs, cuda_stream, zero_fill,
                          zero_fill_count);
        ExampleInfo e;
        e.T = steps;
        e.K = opt.beam_size;
        e.P = dbs_host::pool_size(opt.beam_size, opt.relaxed_pool_multiplier);
        e.V = vocab_size;
        record_decode(handle, e, now_ns() - t0, 1, false);
        clear_error(handle);
        return 0;
    });
}

DBS_EXPORT int dbs_device_decode_batch_variable_ex(
    DBSDecoderHandle* handle, const float* log_probs, int batch_size, int max_steps, int max_beam_size, int vocab_size,
    const int32_t* steps_per_example, const int32_t* beam_sizes_per_example, const int32_t* eos_tokens_per_example,
    const int32_t* min_lengths_per_example, const uint8_t* banned_tokens_per_example,
    const int32_t* forced_tokens_per_example, float repetition_penalty, int no_repeat_ngram_size,
    const DBSDeviceDecodeOutputs* outputs, void* cuda_stream) {
    if (!handle || !log_probs || !outputs || batch_size <= 0 || max_steps <= 0 || max_beam_size <= 0 ||
        vocab_size <= 0) {
        set_error(handle, "invalid variable batch decode arguments");
        mark_error(handle, 1);
        return -1;
    }
    return guarded(handle, [&]() {
        const int64_t t0 = now_ns();
        const size_t B = static_cast<size_t>(batch_size);
        const std::vector<int32_t> forced_h = host_copy(
            forced_tokens_per_example, forced_tokens_per_example ? B * static_cast<size_t>(max_steps) : 0);
        const int64_t stride = static_cast<int64_t>(max_steps) * max_beam_size * vocab_size;
        std::vector<ExampleSpec> spec(B);
        for (size_t b = 0; b < B; ++b) {
            const int steps = steps_per_example ? steps_per_example[b] : max_steps;
            const int beam = beam_sizes_per_example ? beam_sizes_per_example[b] : handle->beam_size;
            if (steps <= 0 || steps > max_steps) throw std::invalid_argument("invalid per-example steps");
            if (beam <= 0 || beam > max_beam_size) throw std::invalid_argument("invalid per-example beam size");
            Options eopt = handle->options;
            eopt.beam_size = beam;
            if (eos_tokens_per_example) eopt.eos_token = eos_tokens_per_example[b];
            if (min_lengths_per_example) eopt.min_length = std::max(0, min_lengths_per_example[b]);
            check_options(eopt);
            const int32_t* fh = forced_tokens_per_example ? forced_h.data() + b * max_steps : nullptr;
            check_example(eopt, log_probs, steps, vocab_size, beam, eopt.eos_token, fh);
            const int cmin = min_lengths_per_example ? min_lengths_per_example[b] : -1;
            spec[b].T = steps;
            spec[b].K = beam;
            spec[b].k_stride = max_beam_size;
            spec[b].x_offset = stride * static_cast<int64_t>(b);
            spec[b].eos = eopt.eos_token;
            spec[b].min_length = cmin >= 0 ? cmin : eopt.min_length;
            spec[b].banned = banned_tokens_per_example ? banned_tokens_per_example + b * static_cast<size_t>(vocab_size)
                                                       : nullptr;
            spec[b].forced = forced_tokens_per_example ? forced_tokens_per_example + b * static_cast<size_t>(max_steps)
                                                       : nullptr;
        }
        CallConstraints cons;
        cons.repetition_penalty = repetition_penalty > 0.0f ? repetition_penalty : 1.0f;
        cons.no_repeat_ngram = no_repeat_ngram_size;
        run_device_decode(handle, log_probs, vocab_size, spec, cons, outputs, cuda_stream);
        ExampleInfo e;
        e.T = spec[0].T;
        e.K = spec[0].K;
        e.P = dbs_host::pool_size(e.K, handle->options.relaxed_pool_multiplier);
        e.V = vocab_size;
        record_decode(handle, e, now_ns() - t0, 1, false);
        clear_error(handle);
        return 0;
    });
}

DBS_EXPORT int dbs_device_backward_batch_ex(DBSDecoderHandle* handle, int batch_size, int steps, int vocab_size,
                                            const DBSDeviceDecodeOutputs* trace, const float* grad_selected_weights,
                                            const float* grad_relaxed_weights, const float* grad_final_scores,
                                            float* grad_log_probs, int64_t* sparse_indices, float* sparse_values,
                                            int64_t* sparse_counts, float* grad_initial_scores, int flags,
                                            void* cuda_stream);

DBS_EXPORT int dbs_device_backward_batch(DBSDecoderHandle* handle, int batch_size, int steps, int vocab_size,
                                         const DBSDeviceDecodeOutputs* trace, const float* grad_selected_weights,
                                         const float* grad_relaxed_weights, const float* grad_final_scores,
                                         float* grad_log_probs, int64_t* sparse_indices, float* sparse_values,
                                         int64_t* sparse_counts, float* grad_initial_scores, void* cuda_stream) {
    return dbs_device_backward_batch_ex(handle, batch_size, steps, vocab_size, trace, grad_selected_weights,
                                        grad_relaxed_weights, grad_final_scores, grad_log_probs, sparse_indices,
                                        sparse_values, sparse_counts, grad_initial_scores, 0, cuda_stream);
}

DBS_EXPORT int dbs_device_backward_batch_ex(DBSDecoderHandle* handle, int batch_size, int steps, int vocab_size,
                                            const DBSDeviceDecodeOutputs* trace, const float* grad_selected_weights,
                                            const float* grad_relaxed_weights, const float* grad_final_scores,
                                            float* grad_log_probs, int64_t* sparse_indices, float* sparse_values,
                                            int64_t* sparse_counts, float* grad_initial_scores, int flags,
                                            void* cuda_stream) {
    if (!handle || !trace) {
        set_error(handle, "invalid decoder or trace pointer");
        return -1;
    }
    return guarded(handle, [&]() {
        const int64_t t0 = now_ns();
        const Options& opt = handle->options;
        if (batch_size <= 0 || steps <= 0 || vocab_size <= 0)
            throw std::invalid_argument("backward dimensions must be positive");
        const bool sparse = sparse_indices != nullptr;
        if (sparse == (grad_log_probs != nullptr))
            throw std::invalid_argument("give exactly one of a dense gradient or sparse outputs");
        if (sparse && (!sparse_values || !sparse_counts))
            throw std::invalid_argument("sparse outputs need indices, values and counts");
        if (grad_selected_weights && !trace->weights)
            throw std::invalid_argument("grad_selected_weights needs the selected weights of the trace");
        if (grad_relaxed_weights && (!trace->relaxed_weights || !trace->pool_parents))
            throw std::invalid_argument("grad_relaxed_weights needs the relaxed pool of the trace");
        std::vector<ExampleSpec> spec(static_cast<size_t>(batch_size));
        for (int b = 0; b < batch_size; ++b) {
            spec[b].T = steps;
            spec[b].K = opt.beam_size;
        }
        const Layout L = dbs_host::make_layout(opt, spec, vocab_size);
        dbs_host::BackwardInputs in;
        in.parents = trace->parents;
        in.tokens = trace->tokens;
        in.lengths = trace->lengths;
        in.weights = trace->weights;
        in.from_logprob = trace->from_logprob;
        in.pool_parents = trace->pool_parents;
        in.pool_tokens = trace->pool_tokens;
        in.pool_lengths = trace->pool_lengths;
        in.relaxed_weights = trace->relaxed_weights;
        in.pool_from_logprob = trace->pool_from_logprob;
        in.grad_selected = grad_selected_weights;
        in.grad_relaxed = grad_relaxed_weights;
        in.grad_final = grad_final_scores;
        dbs_host::BackwardOutputs bo;
        bo.grad_dense = grad_log_probs;
        bo.sparse_indices = sparse_indices;
        bo.sparse_values = sparse_values;
        bo.sparse_counts = sparse_counts;
        bo.grad_initial = grad_initial_scores;
        dbs_host::backward(opt, vocab_size, spec, L, in, bo, static_cast<cudaStream_t>(cuda_stream),
                           (flags & DBS_DEVICE_GRAD_PREZEROED) == 0);
        {
            std::lock_guard<std::mutex> lock(handle->stats_mutex);
            handle->stats.used_sparse_backward = sparse ? 1 : 0;
            handle->stats.used_dense_backward = sparse ? 0 : 1;
            handle->stats.last_backward_ns = now_ns() - t0;
        }
        clear_error(handle);
        return 0;
    });
}

// Uniform-batch example specs of the device entry points.
static std::vector<ExampleSpec> uniform_spec(const Options& opt, int batch_size, int steps, int vocab_size) {
    const int64_t stride = static_cast<int64_t>(steps) * opt.beam_size * vocab_size;
    std::vector<ExampleSpec> spec(static_cast<size_t>(batch_size));
    for (int b = 0; b < batch_size; ++b) {
        spec[b].T = steps;
        spec[b].K = opt.beam_size;
        spec[b].k_stride = opt.beam_size;
        spec[b].x_offset = stride * b;
        spec[b].eos = opt.eos_token;
        spec[b].min_length = opt.min_length;
    }
    return spec;
}

DBS_EXPORT int dbs_device_row_list_capacity(DBSDecoderHandle* handle, int with_pool, int* capacity) {
    if (!handle || !capacity) {
        set_error(handle, "invalid decoder or output pointer");
        return -1;
    }
    return guarded(handle, [&]() {
        *capacity = dbs_host::list_capacity(handle->options, handle->options.beam_size, with_pool != 0, false);
        clear_error(handle);
        return 0;
    });
}

DBS_EXPORT int dbs_device_scan_rows(DBSDecoderHandle* handle, const float* log_probs, int batch_size, int steps,
                                    int vocab_size, int with_pool, int64_t row_begin, int64_t row_end,
                                    uint64_t* lists, int32_t* list_counts, float* list_bounds, void* cuda_stream) {
    if (!handle || !lists || !list_counts || !list_bounds) {
        set_error(handle, "invalid decoder or row list pointer");
        return -1;
    }
    return guarded(handle, [&]() {
        const Options& opt = handle->options;
        if (batch_size <= 0) throw std::invalid_argument("batch_size must be positive");
        check_example(opt, log_probs, steps, vocab_size, opt.beam_size, opt.eos_token, nullptr);
        const int64_t rows = static_cast<int64_t>(batch_size) * steps * opt.beam_size;
        if (row_begin < 0 || row_end < row_begin || row_end > rows)
            throw std::invalid_argument("row range outside the batch's rows");
        const std::vector<ExampleSpec> spec = uniform_spec(opt, batch_size, steps, vocab_size);
        const Layout L = dbs_host::make_layout(opt, spec, vocab_size);
        dbs_host::DecodeControl ctl;
        ctl.synchronize = false;
        ctl.lists = lists;
        ctl.list_count = list_counts;
        ctl.list_bound = list_bounds;
        ctl.scan_begin = row_begin;
        ctl.scan_end = row_end;
        ctl.merge = false;
        dbs_host::Outputs none{};
        dbs_host::decode(opt, log_probs, vocab_size, spec, CallConstraints{}, none, L, with_pool != 0, false,
                         static_cast<cudaStream_t>(cuda_stream), nullptr, ctl);
        clear_error(handle);
        return 0;
    });
}

DBS_EXPORT int dbs_device_merge_rows(DBSDecoderHandle* handle, const float* log_probs, int batch_size, int steps,
                                     int vocab_size, const uint64_t* lists, const int32_t* list_counts,
                                     const float* list_bounds, const DBSDeviceDecodeOutputs* outputs,
                                     void* cuda_stream) {
    if (!handle || !outputs || !lists || !list_counts || !list_bounds) {
        set_error(handle, "invalid decoder, row list or output pointer");
        return -1;
    }
    return guarded(handle, [&]() {
        const Options& opt = handle->options;
        if (batch_size <= 0) throw std::invalid_argument("batch_size must be positive");
        check_example(opt, log_probs, steps, vocab_size, opt.beam_size, opt.eos_token, nullptr);
        dbs_host::DecodeControl ctl;
        ctl.lists = const_cast<uint64_t*>(lists);   // read only when scan is off
        ctl.list_count = const_cast<int32_t*>(list_counts);
        ctl.list_bound = const_cast<float*>(list_bounds);
        ctl.scan = false;
        run_device_decode(handle, log_probs, vocab_size, uniform_spec(opt, batch_size, steps, vocab_size),
                          CallConstraints{}, outputs, cuda_stream, nullptr, 0, &ctl);
        clear_error(handle);
        return 0;
    });
}

DBS_EXPORT int dbs_device_backward_sparse_noalloc(DBSDecoderHandle* handle, int batch_size, int steps,
                                                  int vocab_size, const DBSDeviceDecodeOutputs* trace,
                                                  const float* grad_selected_weights,
                                                  const float* grad_relaxed_weights,
                                                  const float* grad_final_scores, int64_t* sparse_indices,
                                                  float* sparse_values, int64_t* sparse_counts,
                                                  float* grad_initial_scores, void* cuda_stream) {
    if (!handle || !trace) {
        set_error(handle, "invalid decoder or trace pointer");
        return -1;
    }
    return guarded(handle, [&]() {
        const Options& opt = handle->options;
        if (batch_size <= 0 || steps <= 0 || vocab_size <= 0)
            throw std::invalid_argument("backward dimensions must be positive");
        if (!sparse_indices || !sparse_values || !sparse_counts)
            throw std::invalid_argument("sparse outputs need indices, values and counts");
        if (grad_selected_weights && !trace->weights)
            throw std::invalid_argument("grad_selected_weights needs the selected weights of the trace");
        if (grad_relaxed_weights && (!trace->relaxed_weights || !trace->pool_parents))
            throw std::invalid_argument("grad_relaxed_weights needs the relaxed pool of the trace");
        dbs_host::BackwardInputs in;
        in.parents = trace->parents;
        in.tokens = trace->tokens;
        in.lengths = trace->lengths;
        in.weights = trace->weights;
        in.from_logprob = trace->from_logprob;
        in.pool_parents = trace->pool_parents;
        in.pool_tokens = trace->pool_tokens;
        in.pool_lengths = trace->pool_lengths;
        in.relaxed_weights = trace->relaxed_weights;
        in.pool_from_logprob = trace->pool_from_logprob;
        in.grad_selected = grad_selected_weights;
        in.grad_relaxed = grad_relaxed_weights;
        in.grad_final = grad_final_scores;
        dbs_host::BackwardOutputs bo;
        bo.sparse_indices = sparse_indices;
        bo.sparse_values = sparse_values;
        bo.sparse_counts = sparse_counts;
        bo.grad_initial = grad_initial_scores;
        dbs_host::backward_sparse_noalloc(opt, vocab_size, batch_size, steps, in, bo,
                                          static_cast<cudaStream_t>(cuda_stream));
        clear_error(handle);
        return 0;
    });
}

DBS_EXPORT int dbs_device_profile(int enable) {
    try {
        if (enable < 0) {
            dbs_host::profile_reset();
        } else {
            dbs_host::profile_enable(enable != 0 ? ((1u << dbs_host::kProfiledKernels) - 1u) : 0u);
        }
        return 0;
    } catch (...) {
        return -2;
    }
}

DBS_EXPORT int dbs_device_profile_kernels(unsigned mask) {
    try {
        dbs_host::profile_enable(mask & ((1u << dbs_host::kProfiledKernels) - 1u));
        return 0;
    } catch (...) {
        return -2;
    }
}

DBS_EXPORT int dbs_device_profile_read(int kernel, double* total_ms, int64_t* launches) {
    if (!total_ms || !launches) return -1;
    long long n = 0;
    dbs_host::profile_read(kernel, total_ms, &n);
    *launches = n;
    return 0;
}

DBS_EXPORT int dbs_device_last_rescan_counts(DBSDecoderHandle* handle, int64_t* row_rescans, int64_t* merge_rescans) {
    if (!handle) return -1;
    unsigned long long merge = 0, rows = 0;
    dbs_host::last_decode_diagnostics(&merge, nullptr, &rows);
    if (row_rescans) *row_rescans = static_cast<int64_t>(rows);
    if (merge_rescans) *merge_rescans = static_cast<int64_t>(merge);
    return 0;
}

DBS_EXPORT int dbs_device_kernel_launches(int64_t* count) {
    if (!count) return -1;
    *count = static_cast<int64_t>(dbs_host::kernel_launches());
    return 0;
}

}  // extern "C"
