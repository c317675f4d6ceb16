// Host orchestration of the device engine (see engine.h).
#include "engine.h"

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
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
static float gnmt_host(float alpha, int l) {
    if (alpha == 0.0f) return 1.0f;
    const int ll = l < 1 ? 1 : l;
    return std::pow((5.0f + static_cast<float>(ll)) / 6.0f, alpha);
}
static float reciprocal_host(float v) {
    volatile float one = 1.0f;
    return one / v;
}
static void penalty_tables(float alpha, int lmax, std::vector<float>& pen, std::vector<float>& inv) {
    pen.resize(lmax + 1);
    inv.resize(lmax + 1);
    for (int l = 0; l <= lmax; ++l) {
        pen[l] = gnmt_host(alpha, l);
        inv[l] = reciprocal_host(pen[l]);
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
    int dev;
};
std::mutex g_prof_mu;
unsigned g_prof_mask = 0;   // bit i: time kernel i
std::vector<EventPair> g_prof_pending;
double g_prof_ms[kProfiledKernels] = {0};
long long g_prof_n[kProfiledKernels] = {0};

// Timing events are recycled per device: creating and destroying events
// around every launch costs more host time than the launches themselves.
std::vector<std::pair<int, cudaEvent_t>> g_prof_free;

cudaEvent_t prof_take_event_locked(int dev) {
    for (size_t i = g_prof_free.size(); i-- > 0;) {
        if (g_prof_free[i].first == dev) {
            cudaEvent_t e = g_prof_free[i].second;
            g_prof_free.erase(g_prof_free.begin() + static_cast<std::ptrdiff_t>(i));
            return e;
        }
    }
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return e;
}

void prof_drain_locked() {
    for (EventPair& p : g_prof_pending) {
        float ms = 0.0f;
        if (cudaEventSynchronize(p.b) == cudaSuccess && cudaEventElapsedTime(&ms, p.a, p.b) == cudaSuccess) {
            g_prof_ms[p.kernel] += ms;
            g_prof_n[p.kernel] += 1;
        } else {
            cudaGetLastError();
        }
        g_prof_free.emplace_back(p.dev, p.a);
        g_prof_free.emplace_back(p.dev, p.b);
    }
    g_prof_pending.clear();
}

// Records an event pair around one launch on `stream` when profiling is on.
struct ProfileScope {
    cudaEvent_t a = nullptr, b = nullptr;
    cudaStream_t s;
    int kernel;
    int dev = 0;
    ProfileScope(int k, cudaStream_t stream) : s(stream), kernel(k) {
        std::lock_guard<std::mutex> lock(g_prof_mu);
        if (!((g_prof_mask >> k) & 1u)) return;
        if (cudaGetDevice(&dev) != cudaSuccess) {
            cudaGetLastError();
            return;
        }
        a = prof_take_event_locked(dev);
        b = prof_take_event_locked(dev);
        if (!a || !b) {
            if (a) g_prof_free.emplace_back(dev, a);
            if (b) g_prof_free.emplace_back(dev, b);
            a = b = nullptr;
            return;
        }
        cudaEventRecord(a, s);
    }
    ~ProfileScope() {
        if (!a) return;
        cudaEventRecord(b, s);
        std::lock_guard<std::mutex> lock(g_prof_mu);
        g_prof_pending.push_back(EventPair{a, b, kernel, dev});
        if (g_prof_pending.size() >= 65536) prof_drain_locked();  // bound memory when left on
    }
};

// Host-side phase timing of one call, printed to stderr when the environment
// variable DBS_HOST_TRACE is set (read once). Costs one branch otherwise.
struct HostTrace {
    const char* what;
    bool on;
    std::chrono::steady_clock::time_point t0, last;
    std::string line;
    explicit HostTrace(const char* w) : what(w) {
        static const bool enabled = std::getenv("DBS_HOST_TRACE") != nullptr;
        on = enabled;
        if (on) t0 = last = std::chrono::steady_clock::now();
    }
    // DBS_HOST_TRACE=<us> prints only calls slower than that many microseconds
    static double threshold_us() {
        static const double t = [] {
            const char* v = std::getenv("DBS_HOST_TRACE");
            return v ? std::atof(v) : 0.0;
        }();
        return t;
    }
    void mark(const char* label) {
        if (!on) return;
        const auto now = std::chrono::steady_clock::now();
        const double us = std::chrono::duration<double, std::micro>(now - last).count();
        char buf[96];
        std::snprintf(buf, sizeof(buf), " | %s +%.1fus", label, us);
        line += buf;
        last = now;
    }
    ~HostTrace() {
        if (!on) return;
        const double us = std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t0).count();
        if (us >= threshold_us()) std::fprintf(stderr, "[dbs %s] %.1fus%s\n", what, us, line.c_str());
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

// Reusable per-device workspace: a device buffer, a pinned host staging buffer
// (metadata uploads and status read-back go through it, so the copies are
// truly asynchronous) and an event marking the end of the last call that used
// it. Slots grow on demand and are never released before process exit, so a
// steady stream of calls allocates nothing.
struct Slot {
    int device = -1;
    void* dev = nullptr;
    size_t dev_bytes = 0;
    char* pinned = nullptr;
    size_t pinned_bytes = 0;
    cudaEvent_t done = nullptr;
    cudaEvent_t validated = nullptr;   // input validation status has reached the staging buffer
    bool in_use = false;
    // counters of an asynchronous decode, read back into the staging buffer
    const unsigned long long* pending = nullptr;
};

std::atomic<unsigned long long> g_last_merge_rescans{0};
std::atomic<unsigned long long> g_last_row_rescans{0};
std::atomic<unsigned long long> g_timeouts{0};

// Reads the counters an asynchronous decode left in the slot (its event has
// completed); a device wait timeout surfaces here as an error.
void settle(Slot* s) {
    if (!s->pending) return;
    const unsigned long long merge = s->pending[1];
    const unsigned long long timeout = s->pending[3];
    g_last_row_rescans.store(s->pending[0]);
    s->pending = nullptr;
    g_last_merge_rescans.store(merge);
    if (timeout) {
        g_timeouts.fetch_add(1);
        throw CudaFailure("an earlier asynchronous decode reported a device wait timeout");
    }
}

class Arena {
  public:
    Slot* acquire(size_t dev_bytes, size_t pinned_bytes) {
        int device = 0;
        check_cuda(cudaGetDevice(&device), "cudaGetDevice");
        Slot* s = nullptr;
        {
            std::lock_guard<std::mutex> lock(mu_);
            // Prefer an idle slot whose last use has finished and that is
            // already large enough (the smallest such), then the largest idle
            // finished one: calls of different sizes (a decode and its
            // backward) alternating over the slots must not free and
            // reallocate a workspace on every call.
            Slot* fit = nullptr;
            Slot* big = nullptr;
            Slot* busy = nullptr;
            for (Slot* c : slots_) {
                if (c->device != device || c->in_use) continue;
                if (cudaEventQuery(c->done) != cudaSuccess) {
                    cudaGetLastError();
                    if (!busy) busy = c;
                    continue;
                }
                if (c->dev_bytes >= dev_bytes && c->pinned_bytes >= pinned_bytes) {
                    if (!fit || c->dev_bytes < fit->dev_bytes) fit = c;
                } else if (!big || c->dev_bytes > big->dev_bytes) {
                    big = c;
                }
            }
            s = fit ? fit : (big ? big : busy);
            // a new slot rather than waiting for a busy one or growing a small one
            if (!s || ((s == busy || s->dev_bytes < dev_bytes || s->pinned_bytes < pinned_bytes) &&
                       count_on(device) < kMaxSlots)) {
                cudaGetLastError();
                s = new Slot;
                s->device = device;
                check_cuda(cudaEventCreateWithFlags(&s->done, cudaEventDisableTiming), "cudaEventCreate");
                check_cuda(cudaEventCreateWithFlags(&s->validated, cudaEventDisableTiming), "cudaEventCreate");
                slots_.push_back(s);
            }
            s->in_use = true;
        }
        // the host writes the staging buffer below: the previous use must be over
        check_cuda(cudaEventSynchronize(s->done), "workspace reuse");
        try {
            settle(s);
        } catch (...) {
            std::lock_guard<std::mutex> lock(mu_);
            s->in_use = false;
            throw;
        }
        if (s->dev_bytes < dev_bytes) {
            if (s->dev) check_cuda(cudaFree(s->dev), "cudaFree(workspace)");
            s->dev = nullptr;
            s->dev_bytes = 0;
            const size_t n = std::max(dev_bytes + dev_bytes / 4, static_cast<size_t>(1) << 20);
            check_cuda(cudaMalloc(&s->dev, n), "cudaMalloc(workspace)");
            s->dev_bytes = n;
        }
        if (s->pinned_bytes < pinned_bytes) {
            if (s->pinned) check_cuda(cudaFreeHost(s->pinned), "cudaFreeHost(staging)");
            s->pinned = nullptr;
            s->pinned_bytes = 0;
            const size_t n = std::max(pinned_bytes + pinned_bytes / 4, static_cast<size_t>(64) << 10);
            check_cuda(cudaHostAlloc(reinterpret_cast<void**>(&s->pinned), n, cudaHostAllocDefault),
                       "cudaHostAlloc(staging)");
            s->pinned_bytes = n;
        }
        return s;
    }
    void release(Slot* s, cudaStream_t stream) {
        cudaEventRecord(s->done, stream);
        std::lock_guard<std::mutex> lock(mu_);
        s->in_use = false;
    }

  private:
    static constexpr int kMaxSlots = 4;
    int count_on(int device) const {
        int n = 0;
        for (const Slot* c : slots_) n += c->device == device;
        return n;
    }
    std::mutex mu_;
    std::vector<Slot*> slots_;
};

Arena& arena() {
    static Arena* a = new Arena;  // intentionally leaked: outlives static destructors
    return *a;
}

// RAII lease of a slot for one call on one stream.
struct Lease {
    Slot* s;
    cudaStream_t stream;
    Lease(size_t dev_bytes, size_t pinned_bytes, cudaStream_t st) : s(arena().acquire(dev_bytes, pinned_bytes)), stream(st) {}
    ~Lease() { arena().release(s, stream); }
    Lease(const Lease&) = delete;
    Lease& operator=(const Lease&) = delete;
};

// Per-device helper stream and events for work that runs beside the step
// merge (the dense gradient zero fill).
struct Helper {
    cudaStream_t side = nullptr;
    cudaEvent_t before = nullptr;
    cudaEvent_t after = nullptr;
    std::vector<cudaEvent_t> seg;   // end of each row-scan segment of a pipelined decode
};
std::mutex g_helper_mu;
std::vector<Helper> g_helpers;

Helper& helper_locked() {
    int dev = 0;
    check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev >= static_cast<int>(g_helpers.size())) g_helpers.resize(dev + 1);
    Helper& h = g_helpers[dev];
    if (!h.side) {
        check_cuda(cudaStreamCreateWithFlags(&h.side, cudaStreamNonBlocking), "cudaStreamCreate(helper)");
        check_cuda(cudaEventCreateWithFlags(&h.before, cudaEventDisableTiming), "cudaEventCreate");
        check_cuda(cudaEventCreateWithFlags(&h.after, cudaEventDisableTiming), "cudaEventCreate");
    }
    return h;
}

}  // namespace

void last_decode_diagnostics(unsigned long long* merge_rescans, unsigned long long* timeouts,
                             unsigned long long* row_rescans) {
    if (merge_rescans) *merge_rescans = g_last_merge_rescans.load();
    if (row_rescans) *row_rescans = g_last_row_rescans.load();
    if (timeouts) *timeouts = g_timeouts.load();
}

long long kernel_launches() { return dbs_dev::kernel_launch_count(); }

void profile_enable(unsigned mask) {
    std::lock_guard<std::mutex> lock(g_prof_mu);
    g_prof_mask = mask;
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

// A row can contribute at most N candidates, so C = N (+ slack for the
// penalty / n-gram masks) never needs the merge's rescan path; when
// K * (N + slack) exceeds the merge's per-step candidate capacity the lists
// are cut to the capacity and the merge proves per step that nothing dropped
// could have entered (rescanning the row from HBM otherwise), which stays
// exact.
static int list_capacity_for(int N, int K, bool dynamic) {
    const int slack = dynamic ? 8 + N / 8 : 0;
    int C = N + slack;
    if (static_cast<int64_t>(K) * C > dbs_dev::kMaxMergeCandidates) C = std::max(1, dbs_dev::kMaxMergeCandidates / K);
    return C;
}

int list_capacity(const Options& opt, int K, bool pool, bool dynamic) {
    const int P = pool_size(K, opt.relaxed_pool_multiplier);
    return list_capacity_for(pool ? P : K, K, dynamic);
}

// Short row lists for relaxed-pool decodes of many examples. A step's pool
// (P = 8K by default) is spread over the beams' rows: on log_softmax(N(0,1))
// rows of 50257 tokens a row holds more than 64 of a step's pool entries
// about 0.3 times per step at K = 32 (0.8 at K = 64, 1.8 at K = 128). Lists
// of 64 entries keep the row scan near the copy rate (5.4 TB/s against
// 3.5 TB/s with 256-entry lists); the merge proves every other row per step
// and rescans the few that could hold more from HBM, so the selection stays
// exact. Step 0 has one live row, which holds the whole pool: it gets a list
// of up to min(P, 64*K, 1024) entries in the list space of step 0's rows (the other beams'
// rows at step 0 are never extended). The saving grows with the rows a
// call scans (the speculative scan needs many rows per warp) while the
// rescans cost each example's merge a fixed time, and the merges of many
// examples run side by side; so short lists need at least 32 examples and
// 64K rows (measured with T = 64: K = 32, 256 examples 33.5 -> 22.2 ms and
// 32 examples 5.8 -> 4.9 ms; K = 64, 128 examples 25.8 -> 22.5 ms; but
// K = 16 with 32 examples, 32K rows, 2.73 -> 2.88 ms).
constexpr int kFusedMaxExamples = 64;
// Fused decode: DBS_FUSED=0 turns it off; DBS_FUSED_MERGE_CTAS=<n> sets how
// many CTAs merge (default: one per example up to 16 examples, 16 above; a
// CTA with several examples merges them one step at a time in turn, and
// every SM it leaves runs the scan). Measured with T = 64, K = 32,
// V = 50257 (ms per decode + backward, with the merge's prefetch): 32
// examples 3.2-3.3 / 3.14-3.19 / 3.07-3.09 / 3.71-3.73 with 24 / 20 / 16 /
// 14 merge CTAs (14: three examples on some CTAs), 64 examples 5.95 /
// 5.78 / 5.64 / 6.18.
bool fused_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("DBS_FUSED");
        return !(v && std::atoi(v) == 0);
    }();
    return on;
}
int fused_merge_ctas(int B) {
    static const int n = [] {
        const char* v = std::getenv("DBS_FUSED_MERGE_CTAS");
        return v ? std::max(1, std::atoi(v)) : 0;
    }();
    if (n > 0) return std::min(B, n);
    return std::min(B, 16);
}
constexpr int kShortListEntries = 64;
constexpr int kBeam0Extra = 128;
constexpr int kShortListMinExamples = 32;
constexpr int64_t kShortListMinRows = 65536;

void decode(const Options& opt, const float* d_x, int V, const std::vector<ExampleSpec>& ex,
            const CallConstraints& cons, const Outputs& out, const Layout& layout, bool pool,
            bool weights, cudaStream_t stream, DecodeStats* stats, const DecodeControl& ctl) {
    const int B = static_cast<int>(ex.size());
    if (B <= 0) return;
    HostTrace trace("decode");
    const bool dynamic = cons.repetition_penalty > 1.0f || cons.no_repeat_ngram > 0 || ctl.force_seq;

    const bool ext_lists = ctl.lists != nullptr;
    bool short_lists = false;
    if (pool && !dynamic && !ext_lists && B >= kShortListMinExamples && ctl.scan && ctl.merge &&
        ctl.t_begin <= 0 && !ctl.merge_state && !ctl.row_allow) {
        int kmax = 0;
        int64_t nrows = 0;
        bool cut = false;   // some example's full list would be longer
        for (const ExampleSpec& e : ex) {
            kmax = std::max(kmax, e.K);
            nrows += static_cast<int64_t>(e.T) * e.K;
            const int N = pool_size(e.K, opt.relaxed_pool_multiplier);
            cut = cut || list_capacity_for(N, e.K, false) > kShortListEntries;
        }
        // (calls whose merge would be the ranking merge keep full lists)
        short_lists = cut && nrows >= kShortListMinRows && static_cast<int64_t>(kmax) * kShortListEntries > 256;
    }

    // Fused decode: a uniform batch of 2 to kFusedMaxExamples examples without
    // sequence constraints whose merge is the selection merge runs its row
    // scan and its step merge in one cooperative launch (dbs_kernels.cu,
    // fused_decode_kernel), with row lists of at most 64 entries; the merge
    // lists step 0's one live row by a rescan, so no step-0 launch runs.
    // The merge CTAs hold whole SMs, and the row scan's rate is set by the
    // SMs it runs on (it is issue-bound there), so larger batches, whose
    // merges cost less than a tenth of their scan, keep separate launches
    // (measured with T = 64, K = 32, V = 50257: 32 examples 5.07 -> 3.81 ms,
    // 64 examples 7.28 -> 6.87 ms, but 128 examples 11.8 -> 13.0 ms).
    bool fused = false;
    int fused_C = 0;
    if (B <= kFusedMaxExamples && !dynamic && !ext_lists && ctl.scan && ctl.merge && ctl.t_begin <= 0 && ctl.t_end >= (1 << 30) &&
        !ctl.merge_state && !ctl.row_allow && !ctl.x16 && ctl.scan_begin <= 0 && ctl.scan_end < 0 &&
        !(ctl.zero_fill && ctl.zero_fill_count > 0) && fused_enabled()) {
        bool uni = true;
        for (const ExampleSpec& e : ex) uni = uni && e.T == ex[0].T && e.K == ex[0].K;
        const int K0 = ex[0].K;
        const int N0 = pool ? pool_size(K0, opt.relaxed_pool_multiplier) : K0;
        // lists of 64 when many rows share the work (the merge rescans the
        // few rows that hold more of a step's pool), up to 128 for a few
        // examples, whose rows are long per warp and whose rescans would sit
        // on the one merge CTA's critical path
        fused_C = std::min(list_capacity_for(N0, K0, false), B >= 8 ? kShortListEntries : 2 * kShortListEntries);
        const int64_t M0 = static_cast<int64_t>(K0) * fused_C;
        fused = uni && ex[0].T >= 2 && M0 > 256 && M0 <= dbs_dev::kListMergeMaxCandidates && N0 <= dbs_dev::kFusedThreads;
    }
    if (fused) short_lists = false;

    std::vector<dbs_dev::ExampleDesc> desc(B);
    std::vector<int64_t> row_prefix(B + 1, 0);
    int max_T = 0, max_K = 0, max_C = 0, max_N = 0, max_P = 0, max_C0 = 0;
    int64_t rows = 0, list_entries = 0;
    for (int b = 0; b < B; ++b) {
        const ExampleSpec& e = ex[b];
        const int P = layout.P[b];
        const int N = pool ? P : e.K;
        int C = list_capacity_for(N, e.K, dynamic);
        if (short_lists && C > kShortListEntries) C = kShortListEntries;
        if (fused && C > fused_C) C = fused_C;
        if (e.K > 1024) throw LengthError("beam_size above 1024 is not supported by the device decoder");
        dbs_dev::ExampleDesc& d = desc[b];
        d.x_offset = e.x_offset;
        d.row_begin = rows;
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
        d.ext0 = 0;
        d.sel_stride = e.K;
        d.pool_stride = P;
        d.sel_t_stride = e.K;
        d.pool_t_stride = P;
        d.eos = e.eos;
        d.min_length = e.min_length;
        d.banned = e.banned;
        d.forced = e.forced;
        rows += static_cast<int64_t>(e.T) * e.K;
        row_prefix[b + 1] = rows;
        max_T = std::max(max_T, e.T);
        max_K = std::max(max_K, e.K);
        max_C = std::max(max_C, C);
        max_C0 = std::max(max_C0, std::min({N, e.K * C, dbs_dev::kStep0ListMax}));   // step-0 list of a short-list decode
        max_N = std::max(max_N, N);
        max_P = std::max(max_P, P);
    }
    if (pool && out.relaxed_weights && max_P > 1024) {
        throw LengthError("relaxed pool above 1024 entries is not supported by the device decoder");
    }
    // Beam 0's rows list up to kBeam0Extra more entries when the merge is the
    // compact merge (the only one that reads them): the best parent's row
    // holds most of a step's pool, and without them it is the row the
    // merge rescans (91 % of the rescans at K = 32, N = 256, C = 64).
    int max_ext = 0;
    if (pool && !dynamic && !ext_lists && ctl.scan && ctl.merge && !ctl.row_allow &&
        (fused || dbs_dev::compact_merge_applies(max_K, max_C, kBeam0Extra, max_N, dynamic, short_lists))) {
        for (dbs_dev::ExampleDesc& d : desc) {
            int ext = std::min(kBeam0Extra, d.N - d.C);
            ext = std::min(ext, dbs_dev::kListMergeMaxCandidates - d.K * d.C);
            // (the fused launch's scan warps hold lists of up to 192 in shared memory)
            if (fused) ext = std::min(ext, 192 - d.C);
            d.ext0 = std::max(0, ext);
            max_ext = std::max(max_ext, d.ext0);
        }
    }
    for (dbs_dev::ExampleDesc& d : desc) {
        d.list_offset = list_entries;
        list_entries += static_cast<int64_t>(d.T) * (static_cast<int64_t>(d.K) * d.C + d.ext0);
    }
    const int lmax = max_T + 1;
    std::vector<float> pen, inv;
    penalty_tables(opt.length_penalty_alpha, lmax, pen, inv);

    // Workspace layout: [header: desc | row prefix | pen | inv_pen | status |
    // counters] [lists | counts | bounds | prefixes]. The header is staged in
    // pinned memory (status and counters zeroed there) and uploaded with one
    // asynchronous copy.
    const int64_t scan_begin = std::max<int64_t>(0, ctl.scan_begin);
    const int64_t scan_end = ctl.scan_end < 0 ? rows : std::min<int64_t>(rows, ctl.scan_end);
    // One example whose merge is the selection merge (one CTA, T dependent
    // steps, the slow half of such a decode): the row scan runs in segments
    // of steps on the helper stream, and each segment's merge starts as soon
    // as its rows are listed, beside the scan of the next segment; the beam
    // state passes between the merge launches in the workspace.
    int seg_steps = 0, n_seg = 0;
    if (!fused && B == 1 && ctl.scan && ctl.merge && !ext_lists && scan_begin == 0 && scan_end == rows &&
        ctl.t_begin <= 0 && ctl.t_end >= max_T && !ctl.merge_state && !ctl.row_allow && max_T >= 32 &&
        (dynamic || static_cast<int64_t>(max_K) * max_C > 256)) {
        // about 512 rows per segment (at least 16 steps): the first merge
        // starts after one short scan, and a segment's scan (each warp near
        // its own streaming limit) stays ahead of its merge
        seg_steps = std::max(16, std::min(max_T, 512 / std::max(1, max_K)));
        n_seg = (max_T + seg_steps - 1) / seg_steps;
        if (n_seg < 2) n_seg = 0;
    }
    const bool pipeline = n_seg > 0;
    size_t hdr = 0;
    hdr += bytes_of<dbs_dev::ExampleDesc>(B);
    hdr += bytes_of<int64_t>(B + 1);
    hdr += 2 * bytes_of<float>(lmax + 1);
    hdr += bytes_of<int32_t>(B);
    hdr += bytes_of<unsigned long long>(4);
    if (pipeline) hdr += bytes_of<unsigned long long>(n_seg);   // first row of each scan segment
    if (ext_lists && (!ctl.list_count || !ctl.list_bound)) throw InvalidArgument("row lists need counts and bounds");
    if (!ext_lists && !(ctl.scan && ctl.merge)) throw InvalidArgument("a split decode needs caller row lists");
    size_t ws = hdr;
    if (!ext_lists) {
        ws += bytes_of<uint64_t>(static_cast<size_t>(list_entries));
        ws += bytes_of<int32_t>(static_cast<size_t>(rows));
        ws += bytes_of<float>(static_cast<size_t>(rows));
    }
    if (dynamic && !ctl.seq_scratch) ws += bytes_of<int32_t>(static_cast<size_t>(B) * 3 * max_K * max_T);
    if (pipeline || fused) ws += bytes_of<float>(static_cast<size_t>(4) * max_K * B);   // merge state between segments
    if (fused) ws += bytes_of<unsigned int>(static_cast<size_t>(B) * max_T);   // rows listed per (example, step)
    trace.mark("prepared");
    Lease lease(ws, hdr, stream);
    trace.mark("slot");
    Carve cv{static_cast<char*>(lease.s->dev), 0, ws};
    Carve hv{lease.s->pinned, 0, hdr};

    dbs_dev::DecodeParams p{};
    auto* d_desc = cv.take<dbs_dev::ExampleDesc>(B);
    auto* d_prefix = cv.take<int64_t>(B + 1);
    auto* d_pen = cv.take<float>(lmax + 1);
    auto* d_inv = cv.take<float>(lmax + 1);
    p.status = cv.take<int32_t>(B);
    p.counters = cv.take<unsigned long long>(4);
    std::memcpy(hv.take<dbs_dev::ExampleDesc>(B), desc.data(), sizeof(dbs_dev::ExampleDesc) * B);
    std::memcpy(hv.take<int64_t>(B + 1), row_prefix.data(), sizeof(int64_t) * (B + 1));
    std::memcpy(hv.take<float>(lmax + 1), pen.data(), sizeof(float) * (lmax + 1));
    std::memcpy(hv.take<float>(lmax + 1), inv.data(), sizeof(float) * (lmax + 1));
    int32_t* h_status = hv.take<int32_t>(B);
    unsigned long long* h_counters = hv.take<unsigned long long>(4);
    std::memset(h_status, 0, sizeof(int32_t) * B);
    std::memset(h_counters, 0, sizeof(unsigned long long) * 4);
    h_counters[2] = static_cast<unsigned long long>(scan_begin);   // first row the scan claims
    unsigned long long* h_seeds = nullptr;
    if (pipeline) {
        cv.take<unsigned long long>(n_seg);
        h_seeds = hv.take<unsigned long long>(n_seg);
        for (int i = 0; i < n_seg; ++i)
            h_seeds[i] = static_cast<unsigned long long>(i) * seg_steps * desc[0].K;
    }
    check_cuda(cudaMemcpyAsync(lease.s->dev, lease.s->pinned, cv.off, cudaMemcpyHostToDevice, stream),
               "upload decode metadata");
    if (ext_lists) {
        p.lists = ctl.lists;
        p.list_count = ctl.list_count;
        p.list_bound = ctl.list_bound;
    } else {
        p.lists = cv.take<uint64_t>(static_cast<size_t>(list_entries));
        p.list_count = cv.take<int32_t>(static_cast<size_t>(rows));
        p.list_bound = cv.take<float>(static_cast<size_t>(rows));
    }
    p.seq_scratch = !dynamic ? nullptr
                  : ctl.seq_scratch ? ctl.seq_scratch
                                    : cv.take<int32_t>(static_cast<size_t>(B) * 3 * max_K * max_T);
    float* d_state = (pipeline || fused) ? cv.take<float>(static_cast<size_t>(4) * max_K * B) : nullptr;
    unsigned int* d_done = fused ? cv.take<unsigned int>(static_cast<size_t>(B) * max_T) : nullptr;
    p.t_begin = ctl.t_begin;
    p.t_end = ctl.t_end;
    p.merge_state = ctl.merge_state;
    p.row_allow = ctl.row_allow;
    p.force_seq = ctl.force_seq ? 1 : 0;
    p.first_row_apart = short_lists ? 1 : 0;
    p.first_rows_only = 0;

    p.x = d_x;
    p.x16 = ctl.x16;
    p.x16_bf16 = ctl.x16_bf16 ? 1 : 0;
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

    // status and counters are contiguous in the header: one read-back each time
    const size_t st_off = reinterpret_cast<char*>(p.status) - static_cast<char*>(lease.s->dev);
    const size_t st_bytes = reinterpret_cast<char*>(p.counters + 4) - reinterpret_cast<char*>(p.status);
    const bool validate = opt.validate_inputs && ctl.scan;   // a merge-only call trusts its scan call
    if (validate) {
        // The small validation kernel runs first, on the caller's stream: it
        // takes microseconds alone, whereas beside a persistent row-scan grid
        // it waited for SM room until the scan ended, and the host waits for
        // its verdict before it queues the merge. Its verdict is then back
        // while the scan runs.
        {
            ProfileScope ps(kValidate, stream);
            check_cuda(dbs_dev::launch_validate(p, stream), "validate kernel");
        }
        check_cuda(cudaMemcpyAsync(lease.s->pinned + st_off, p.status, st_bytes, cudaMemcpyDeviceToHost, stream),
                   "read status");
        check_cuda(cudaEventRecord(lease.s->validated, stream), "cudaEventRecord");
    }
    if (pipeline) {
        // Segments of steps: the helper stream seeds the row-claim counter
        // and scans each segment's rows after the validation kernel; the
        // merge of segment i (on `stream`) waits only for scan i, so it runs
        // beside the scans of later segments.
        // seg_done[n_seg]: the helper stream's part of this call is over
        std::vector<cudaEvent_t> seg_done(n_seg + 1, nullptr);
        struct EventsGuard {
            std::vector<cudaEvent_t>& v;
            ~EventsGuard() {
                for (cudaEvent_t e : v)
                    if (e) cudaEventDestroy(e);   // released once the queued waits are done
            }
        } events_guard{seg_done};
        for (cudaEvent_t& ev : seg_done)
            check_cuda(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "cudaEventCreate");
        const int K0 = desc[0].K;
        {
            std::lock_guard<std::mutex> lock(g_helper_mu);
            Helper& hp = helper_locked();
            // the metadata upload, the validation and the caller's earlier work come first
            check_cuda(cudaEventRecord(hp.before, stream), "cudaEventRecord");
            check_cuda(cudaStreamWaitEvent(hp.side, hp.before, 0), "cudaStreamWaitEvent");
            for (int i = 0; i < n_seg; ++i) {
                const int64_t r0 = static_cast<int64_t>(i) * seg_steps * K0;
                const int64_t r1 = std::min<int64_t>(rows, r0 + static_cast<int64_t>(seg_steps) * K0);
                check_cuda(cudaMemcpyAsync(p.counters + 2, h_seeds + i, sizeof(unsigned long long),
                                           cudaMemcpyHostToDevice, hp.side),
                           "seed row claims");
                {
                    ProfileScope ps(kRowScan, hp.side);
                    dbs_dev::DecodeParams ps_p = p;
                    ps_p.total_rows = r1;
                    check_cuda(dbs_dev::launch_row_scan(ps_p, max_C + max_ext, device_sm_count(), hp.side, r1 - r0),
                               "row scan kernel");
                }
                check_cuda(cudaEventRecord(seg_done[i], hp.side), "cudaEventRecord");
            }
            if (ctl.zero_fill && ctl.zero_fill_count > 0) {
                // after the scans, beside the remaining merges
                ProfileScope ps(kFillZero, hp.side);
                check_cuda(dbs_dev::launch_fill_zero_bulk(ctl.zero_fill, ctl.zero_fill_count, device_sm_count(),
                                                          hp.side),
                           "zero fill kernel");
            }
            check_cuda(cudaEventRecord(seg_done[n_seg], hp.side), "cudaEventRecord");
        }
        trace.mark("row scan queued");
        if (validate) {
            check_cuda(cudaEventSynchronize(lease.s->validated), "validate");
            trace.mark("validate synced");
            for (int b = 0; b < B; ++b) {
                if (h_status[b]) {
                    // the workspace is released on `stream`: it must cover the scans
                    check_cuda(cudaStreamWaitEvent(stream, seg_done[n_seg], 0), "cudaStreamWaitEvent");
                    throw InvalidArgument("log_probs contains NaN or +Inf");
                }
            }
        }
        for (int i = 0; i < n_seg; ++i) {
            check_cuda(cudaStreamWaitEvent(stream, seg_done[i], 0), "cudaStreamWaitEvent");
            dbs_dev::DecodeParams mp = p;
            mp.t_begin = i * seg_steps;
            mp.t_end = std::min(max_T, (i + 1) * seg_steps);
            mp.merge_state = d_state;
            ProfileScope ps(kStepMerge, stream);
            check_cuda(dbs_dev::launch_step_merge(mp, max_K, max_C, max_T, max_N, dynamic, stream, 0, max_ext),
                       "step merge kernel");
        }
        trace.mark("merge queued");
        check_cuda(cudaStreamWaitEvent(stream, seg_done[n_seg], 0), "cudaStreamWaitEvent");
    } else if (fused) {
        // merge CTAs: one per example up to 16 examples, else examples in turn
        const int merge_ctas = fused_merge_ctas(B);
        check_cuda(cudaMemsetAsync(d_done, 0, sizeof(unsigned int) * static_cast<size_t>(B) * max_T, stream),
                   "zero step counters");
        dbs_dev::DecodeParams fp = p;
        fp.step_major_bk = static_cast<int64_t>(B) * max_K;
        fp.step_major_tk = static_cast<int64_t>(max_T) * max_K;
        fp.merge_state = d_state;
        cudaError_t ferr;
        {
            ProfileScope ps(kRowScan, stream);   // the whole fused launch
            ferr = dbs_dev::launch_fused_decode(fp, max_K, max_C, max_ext, max_N, merge_ctas, d_done, device_sm_count(),
                                                stream);
        }
        if (ferr == cudaErrorNotSupported) {
            cudaGetLastError();
            // separate launches on the same lists (the merge's rescans list step 0)
            {
                ProfileScope ps(kRowScan, stream);
                check_cuda(dbs_dev::launch_row_scan(p, max_C + max_ext, device_sm_count(), stream, rows), "row scan kernel");
            }
            if (validate) {
                check_cuda(cudaEventSynchronize(lease.s->validated), "validate");
                for (int b = 0; b < B; ++b)
                    if (h_status[b]) throw InvalidArgument("log_probs contains NaN or +Inf");
            }
            ProfileScope ps(kStepMerge, stream);
            check_cuda(dbs_dev::launch_step_merge(p, max_K, max_C, max_T, max_N, dynamic, stream, 0, max_ext), "step merge kernel");
        } else {
            check_cuda(ferr, "fused decode kernel");
            trace.mark("fused queued");
            if (validate) {
                // the fused launch writes no output when validation flagged an
                // example; the call reports the error
                check_cuda(cudaEventSynchronize(lease.s->validated), "validate");
                trace.mark("validate synced");
                for (int b = 0; b < B; ++b)
                    if (h_status[b]) throw InvalidArgument("log_probs contains NaN or +Inf");
            }
        }
    } else {
        if (ctl.scan && scan_end > scan_begin) {
            ProfileScope ps(kRowScan, stream);
            dbs_dev::DecodeParams ps_p = p;
            ps_p.total_rows = scan_end;   // rows are claimed from scan_begin up to here
            check_cuda(dbs_dev::launch_row_scan(ps_p, max_C + max_ext, device_sm_count(), stream, scan_end - scan_begin),
                       "row scan kernel");
            if (short_lists) {
                // the live step-0 row of every example, with its long list
                // (claims restart at 0: claim i is example i's first row)
                check_cuda(cudaMemsetAsync(p.counters + 2, 0, sizeof(unsigned long long), stream),
                           "row claim reset");
                ps_p.first_rows_only = 1;
                check_cuda(dbs_dev::launch_row_scan(ps_p, max_C0, device_sm_count(), stream, B),
                           "row scan kernel (step 0)");
            }
        }
        trace.mark("row scan queued");
        if (validate) {
            // The reference rejects NaN / +Inf before decoding. The row scan is
            // already queued (it only writes this call's workspace and tolerates
            // any value), so the GPU keeps streaming while the host waits for the
            // small validation kernel; nothing that writes an output is queued
            // before the verdict.
            check_cuda(cudaEventSynchronize(lease.s->validated), "validate");
            trace.mark("validate synced");
            for (int b = 0; b < B; ++b)
                if (h_status[b]) throw InvalidArgument("log_probs contains NaN or +Inf");
        }
        if (!ctl.merge) {
            // scan-only call: read the counters back for the timeout check
        } else if (ctl.zero_fill && ctl.zero_fill_count > 0) {
            // zero the gradient buffer on the helper stream while the (latency
            // bound, few-CTA) step merge runs; `stream` waits for it afterwards
            // The merge is queued first; the fill is one 32-thread CTA per SM
            // issuing bulk stores, so merge CTAs always fit beside it and keep
            // the load/store pipe to themselves.
            std::lock_guard<std::mutex> lock(g_helper_mu);
            Helper& hp = helper_locked();
            check_cuda(cudaEventRecord(hp.before, stream), "cudaEventRecord");
            {
                ProfileScope ps(kStepMerge, stream);
                check_cuda(dbs_dev::launch_step_merge(p, max_K, max_C, max_T, max_N, dynamic, stream, 0, max_ext),
                           "step merge kernel");
            }
            trace.mark("merge queued");
            check_cuda(cudaStreamWaitEvent(hp.side, hp.before, 0), "cudaStreamWaitEvent");
            {
                ProfileScope ps(kFillZero, hp.side);
                check_cuda(dbs_dev::launch_fill_zero_bulk(ctl.zero_fill, ctl.zero_fill_count, device_sm_count(), hp.side),
                           "zero fill kernel");
            }
            check_cuda(cudaEventRecord(hp.after, hp.side), "cudaEventRecord");
            trace.mark("fill queued");
            check_cuda(cudaStreamWaitEvent(stream, hp.after, 0), "cudaStreamWaitEvent");
        } else {
            ProfileScope ps(kStepMerge, stream);
            check_cuda(dbs_dev::launch_step_merge(p, max_K, max_C, max_T, max_N, dynamic, stream, 0, max_ext), "step merge kernel");
        }
    }
    const bool want_w = (p.weights && p.scores) || (p.relaxed_weights && p.pool_scores);
    if (want_w && ctl.merge && ctl.weights) {
        ProfileScope ps(kWeights, stream);
        check_cuda(dbs_dev::launch_weights(p, max_T, max_K, max_P, stream), "weights kernel");
    }
    check_cuda(cudaMemcpyAsync(lease.s->pinned + st_off, p.status, st_bytes, cudaMemcpyDeviceToHost, stream),
               "read counters");
    if (ctl.synchronize) {
        check_cuda(cudaStreamSynchronize(stream), "decode");
        if (stats) {
            stats->row_rescans = h_counters[0];
            stats->merge_fallbacks = h_counters[1];
        }
        g_last_merge_rescans.store(h_counters[1]);
        g_last_row_rescans.store(h_counters[0]);
        if (h_counters[3]) {
            g_timeouts.fetch_add(1);
            throw CudaFailure("row scan: a shared-memory copy did not complete within the wait bound");
        }
    } else {
        lease.s->pending = h_counters;
    }
}

void backward(const Options& opt, int V, const std::vector<ExampleSpec>& ex, const Layout& layout,
              const BackwardInputs& in, const BackwardOutputs& out, cudaStream_t stream, bool zero_dense) {
    HostTrace trace("backward");
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
    const size_t hdr = bytes_of<dbs_dev::ExampleDesc>(B) + bytes_of<float>(lmax + 1);
    const size_t ws = hdr + bytes_of<int32_t>(static_cast<size_t>(B) * max_T);
    trace.mark("prepared");
    Lease lease(ws, hdr, stream);
    trace.mark("slot");
    Carve cv{static_cast<char*>(lease.s->dev), 0, ws};
    Carve hv{lease.s->pinned, 0, hdr};
    auto* d_desc = cv.take<dbs_dev::ExampleDesc>(B);
    auto* d_inv = cv.take<float>(lmax + 1);
    std::memcpy(hv.take<dbs_dev::ExampleDesc>(B), desc.data(), sizeof(dbs_dev::ExampleDesc) * B);
    std::memcpy(hv.take<float>(lmax + 1), inv.data(), sizeof(float) * (lmax + 1));
    check_cuda(cudaMemcpyAsync(lease.s->dev, lease.s->pinned, cv.off, cudaMemcpyHostToDevice, stream),
               "upload backward metadata");
    auto* d_steps = cv.take<int32_t>(static_cast<size_t>(B) * max_T);
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
    trace.mark("queued");
}

void backward_sparse_noalloc(const Options& opt, int V, int B, int T, const BackwardInputs& in,
                             const BackwardOutputs& out, cudaStream_t stream) {
    const int K = opt.beam_size;
    const int P = pool_size(K, opt.relaxed_pool_multiplier);
    if (T > dbs_dev::kNoAllocMaxSteps)
        throw LengthError("the allocation-free backward takes at most " + std::to_string(dbs_dev::kNoAllocMaxSteps) +
                          " steps");
    if (static_cast<int64_t>(B) * T > dbs_dev::kNoAllocMaxStepCounts)
        throw LengthError("the allocation-free backward takes at most " +
                          std::to_string(dbs_dev::kNoAllocMaxStepCounts) + " batch_size * steps (its static scratch)");
    if (K + P > dbs_dev::kNoAllocMaxBeamPlusPool)
        throw LengthError("the allocation-free backward takes at most " +
                          std::to_string(dbs_dev::kNoAllocMaxBeamPlusPool) + " beam + pool entries per step");
    float inv[dbs_dev::kNoAllocMaxSteps + 2];
    for (int l = 0; l < T + 2; ++l) inv[l] = reciprocal_host(gnmt_host(opt.length_penalty_alpha, l));
    dbs_dev::BackwardParams p{};
    p.V = V;
    p.B = B;
    p.Lmax = T + 1;
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
    p.sparse_indices = out.sparse_indices;
    p.sparse_values = out.sparse_values;
    p.sparse_counts = out.sparse_counts;
    p.grad_initial = out.grad_initial;
    check_cuda(dbs_dev::launch_backward_noalloc(p, T, K, P, inv, stream), "allocation-free backward kernel");
}

// Filter-free checks that decide whether the reference consults the token
// filter (scan_parent_row_scalar_advanced, src/differentiable_beam.cpp:512-549:
// forced, banned, EOS before min_length, then the n-gram check of
// token_allowed_by_advanced_constraints, :327-351).
static bool ngram_repeats(const std::vector<int32_t>& pre, int n, int token) {
    if (n <= 0) return false;
    if (n == 1) {
        for (int32_t v : pre)
            if (v == token) return true;
        return false;
    }
    const int len = static_cast<int>(pre.size());
    if (len + 1 < n) return false;
    const int suffix = len - (n - 1);
    for (int i = 0; i + n <= len; ++i) {
        bool same = true;
        for (int j = 0; j < n - 1 && same; ++j) same = pre[i + j] == pre[suffix + j];
        if (same && pre[i + n - 1] == token) return true;
    }
    return false;
}

// Device allocation of the filtered decode, released in stream order.
struct StepBuffer {
    void* ptr = nullptr;
    cudaStream_t stream;
    StepBuffer(size_t n, cudaStream_t s) : stream(s) {
        if (n) check_cuda(cudaMallocAsync(&ptr, n, s), "cudaMallocAsync(filtered decode)");
    }
    ~StepBuffer() {
        if (ptr) cudaFreeAsync(ptr, stream);
    }
    StepBuffer(const StepBuffer&) = delete;
    StepBuffer& operator=(const StepBuffer&) = delete;
    template <class T>
    T* as() const { return static_cast<T*>(ptr); }
};

void decode_filtered(const Options& opt, const float* d_x, int V, const ExampleSpec& ex, const uint8_t* h_banned,
                     const int32_t* h_forced, const CallConstraints& cons, const Outputs& out, const Layout& layout,
                     cudaStream_t stream, DecodeStats* stats, const TokenFilter& filter) {
    const int T = ex.T, K = ex.K;
    const bool pool = out.pool_scores != nullptr;
    const int C = list_capacity(opt, K, pool, true);
    const int64_t rows = static_cast<int64_t>(T) * K;
    // state kept between the per-step launches (device) and its host mirror
    StepBuffer lists(static_cast<size_t>(rows) * C * sizeof(uint64_t), stream);
    StepBuffer counts(static_cast<size_t>(rows) * sizeof(int32_t), stream);
    StepBuffer bounds(static_cast<size_t>(rows) * sizeof(float), stream);
    StepBuffer state(static_cast<size_t>(4) * K * sizeof(float), stream);
    StepBuffer seq(static_cast<size_t>(3) * K * T * sizeof(int32_t), stream);
    StepBuffer allow(static_cast<size_t>(K) * V, stream);
    std::vector<uint8_t> h_allow(static_cast<size_t>(K) * V);
    std::vector<float> h_state(static_cast<size_t>(4) * K);
    std::vector<int32_t> h_seq(static_cast<size_t>(K) * T);
    std::vector<std::vector<int32_t>> prefix(K);
    std::vector<float> raw(K, -std::numeric_limits<float>::infinity());
    std::vector<int> len(K, 0), ended(K, 0);
    raw[0] = 0.0f;
    const int min_len = ex.min_length;
    for (int t = 0; t < T; ++t) {
        if (t > 0) {
            // beams after step t-1: state and the prefix buffer of parity t
            check_cuda(cudaMemcpyAsync(h_state.data(), state.ptr, h_state.size() * sizeof(float),
                                       cudaMemcpyDeviceToHost, stream), "read beam state");
            const int32_t* cur = seq.as<int32_t>() + ((t & 1) ? static_cast<size_t>(K) * T : 0);
            check_cuda(cudaMemcpyAsync(h_seq.data(), cur, h_seq.size() * sizeof(int32_t), cudaMemcpyDeviceToHost,
                                       stream), "read beam prefixes");
            check_cuda(cudaStreamSynchronize(stream), "filtered decode step");
            for (int k = 0; k < K; ++k) {
                raw[k] = h_state[k];
                int v = 0;
                std::memcpy(&v, &h_state[K + k], sizeof(int));
                len[k] = v;
                std::memcpy(&v, &h_state[2 * K + k], sizeof(int));
                ended[k] = v;
                std::memcpy(&v, &h_state[3 * K + k], sizeof(int));
                prefix[k].assign(h_seq.begin() + static_cast<size_t>(k) * T, h_seq.begin() + static_cast<size_t>(k) * T + v);
            }
        }
        const int forced = h_forced ? h_forced[t] : -1;
        std::fill(h_allow.begin(), h_allow.end(), uint8_t{0});
        for (int k = 0; k < K; ++k) {
            if (!std::isfinite(raw[k]) || (ex.eos >= 0 && ended[k])) continue;   // not scanned
            const int new_len = len[k] + 1;
            uint8_t* a = h_allow.data() + static_cast<size_t>(k) * V;
            for (int v = 0; v < V; ++v) {
                if (forced >= 0 && v != forced) continue;
                if (h_banned && h_banned[v]) continue;
                if (ex.eos >= 0 && v == ex.eos && new_len < min_len) continue;
                if (ngram_repeats(prefix[k], cons.no_repeat_ngram, v)) continue;
                a[v] = filter(t, k, prefix[k].empty() ? nullptr : prefix[k].data(), static_cast<int>(prefix[k].size()),
                              v) != 0;
            }
        }
        check_cuda(cudaMemcpyAsync(allow.ptr, h_allow.data(), h_allow.size(), cudaMemcpyHostToDevice, stream),
                   "upload filter verdicts");
        DecodeControl ctl;
        ctl.synchronize = true;
        ctl.lists = lists.as<uint64_t>();
        ctl.list_count = counts.as<int32_t>();
        ctl.list_bound = bounds.as<float>();
        ctl.scan_begin = static_cast<int64_t>(t) * K;
        ctl.scan_end = static_cast<int64_t>(t + 1) * K;
        ctl.t_begin = t;
        ctl.t_end = t + 1;
        ctl.merge_state = state.as<float>();
        ctl.seq_scratch = seq.as<int32_t>();
        ctl.row_allow = allow.as<uint8_t>();
        ctl.force_seq = true;
        ctl.weights = t + 1 == T;
        Options step_opt = opt;
        step_opt.validate_inputs = t == 0 ? opt.validate_inputs : 0;
        decode(step_opt, d_x, V, {ex}, cons, out, layout, pool, out.weights != nullptr, stream, stats, ctl);
    }
}

void decode_model_steps(const Options& opt, float* d_x, int V, const ExampleSpec& ex, const Outputs& out,
                        const Layout& layout, cudaStream_t stream, DecodeStats* stats, const StepRows& rows) {
    const int T = ex.T, K = ex.K;
    const bool pool = out.pool_scores != nullptr;
    const int C = list_capacity(opt, K, pool, true);
    const int64_t nrows = static_cast<int64_t>(T) * K;
    StepBuffer lists(static_cast<size_t>(nrows) * C * sizeof(uint64_t), stream);
    StepBuffer counts(static_cast<size_t>(nrows) * sizeof(int32_t), stream);
    StepBuffer bounds(static_cast<size_t>(nrows) * sizeof(float), stream);
    StepBuffer state(static_cast<size_t>(4) * K * sizeof(float), stream);
    StepBuffer seq(static_cast<size_t>(3) * K * T * sizeof(int32_t), stream);
    std::vector<float> h_state(static_cast<size_t>(4) * K);
    std::vector<int32_t> tokens(static_cast<size_t>(K), -1);
    std::vector<float> scores(static_cast<size_t>(K) + 1, 0.0f);
    for (int t = 0; t < T; ++t) {
        if (t > 0) {
            // tokens of step t-1 and the final scores of the decode so far
            // (finalisation, src/differentiable_beam.cpp:1661-1667)
            check_cuda(cudaMemcpyAsync(tokens.data(), out.tokens + static_cast<size_t>(t - 1) * K,
                                       sizeof(int32_t) * K, cudaMemcpyDeviceToHost, stream), "read tokens");
            check_cuda(cudaMemcpyAsync(h_state.data(), state.ptr, h_state.size() * sizeof(float),
                                       cudaMemcpyDeviceToHost, stream), "read beam state");
            check_cuda(cudaStreamSynchronize(stream), "model step");
            for (int k = 0; k < K; ++k) {
                int len = 0;
                std::memcpy(&len, &h_state[K + k], sizeof(int));
                scores[k] = h_state[k] / gnmt_host(opt.length_penalty_alpha, len < 1 ? 1 : len);
            }
        }
        rows(t, tokens.data(), scores.data(), d_x + static_cast<size_t>(t) * K * V);
        DecodeControl ctl;
        ctl.synchronize = true;
        ctl.lists = lists.as<uint64_t>();
        ctl.list_count = counts.as<int32_t>();
        ctl.list_bound = bounds.as<float>();
        ctl.scan_begin = static_cast<int64_t>(t) * K;
        ctl.scan_end = static_cast<int64_t>(t + 1) * K;
        ctl.t_begin = t;
        ctl.t_end = t + 1;
        ctl.merge_state = state.as<float>();
        ctl.seq_scratch = seq.as<int32_t>();
        ctl.force_seq = true;   // the merge that keeps its state between launches
        ctl.weights = t + 1 == T;
        Options step_opt = opt;
        step_opt.validate_inputs = 0;   // rows beyond step t are not written yet; the caller validates
        decode(step_opt, d_x, V, {ex}, CallConstraints{}, out, layout, pool, out.weights != nullptr, stream, stats,
               ctl);
    }
}

}  // namespace dbs_host

