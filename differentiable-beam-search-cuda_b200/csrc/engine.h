// Host side of the device engine: turns a batch of per-example decode specs
// into descriptors, sizes and carves the workspace, and launches the kernels
// of dbs_kernels.cu on one stream.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <functional>
#include <vector>

#include <cuda_runtime.h>

#include "dbs_engine.h"

namespace dbs_host {

// Decoder options after the reference's default substitution
// (from_c_options, src/differentiable_beam.cpp:3145-3177).
struct Options {
    int beam_size = 8;
    int eos_token = -1;
    float selected_temperature = 1.0f;
    float soft_topk_temperature = 0.25f;
    int relaxed_pool_multiplier = 8;
    int vocab_block = 4096;
    float length_penalty_alpha = 0.0f;
    float soft_topk_tolerance = 1.0e-4f;
    int soft_topk_max_iters = 48;
    int min_length = 0;
    int validate_inputs = 1;
    int64_t max_dense_gradient_elements = 100000000LL;
};

int pool_size(int beam_size, int multiplier);

// One example of a decode call. banned / forced are DEVICE pointers.
struct ExampleSpec {
    int T = 0;
    int K = 0;
    int k_stride = 0;            // rows per step in the input layout
    int64_t x_offset = 0;        // element offset of the example in x
    int eos = -1;
    int min_length = 0;          // effective EOS min length
    const uint8_t* banned = nullptr;
    const int32_t* forced = nullptr;
};

// Device output arrays. Selected arrays are tight per example ([T_e, K_e]
// back to back), pool arrays [T_e, P_e] back to back, finals [K_e].
struct Outputs {
    int32_t* parents = nullptr;
    int32_t* tokens = nullptr;
    int32_t* lengths = nullptr;
    float* raw_scores = nullptr;
    float* scores = nullptr;
    float* weights = nullptr;
    uint8_t* from_logprob = nullptr;
    int32_t* pool_parents = nullptr;
    int32_t* pool_tokens = nullptr;
    int32_t* pool_lengths = nullptr;
    float* pool_raw_scores = nullptr;
    float* pool_scores = nullptr;
    float* relaxed_weights = nullptr;
    uint8_t* pool_from_logprob = nullptr;
    float* final_raw_scores = nullptr;
    float* final_scores = nullptr;
};

struct CallConstraints {
    float repetition_penalty = 1.0f;  // > 1 enables
    int no_repeat_ngram = 0;          // > 0 enables
};

// Element counts of the tight per-example output layout.
struct Layout {
    std::vector<int64_t> sel_offset;   // [B]
    std::vector<int64_t> pool_offset;  // [B]
    std::vector<int64_t> final_offset; // [B]
    std::vector<int64_t> grad_offset;  // [B]
    std::vector<int64_t> sparse_offset;// [B]
    std::vector<int> P;                // [B]
    int64_t sel_total = 0;
    int64_t pool_total = 0;
    int64_t final_total = 0;
    int64_t grad_total = 0;
    int64_t sparse_total = 0;
};

Layout make_layout(const Options& opt, const std::vector<ExampleSpec>& ex, int V);

// Thrown for errors the reference reports as std::invalid_argument.
struct InvalidArgument : std::invalid_argument {
    using std::invalid_argument::invalid_argument;
};
struct CudaFailure : std::runtime_error {
    using std::runtime_error::runtime_error;
};
struct LengthError : std::length_error {
    using std::length_error::length_error;
};

void check_cuda(cudaError_t err, const char* what);

// Runs the full forward on `stream`. When `pool` is false only the top-K per
// step is selected (the pool and relaxed weights are not produced); when
// `weights` is false the selected softmax is skipped. Returns after the
// stream has finished; throws InvalidArgument when validation failed.
struct DecodeStats {
    unsigned long long row_rescans = 0;
    unsigned long long merge_fallbacks = 0;
};

// How a decode call meets the host. Validation (when enabled) is always
// checked before the heavy kernels are launched: the call waits for the small
// validation kernel only. With `synchronize` the call also waits for the
// whole decode (host mirrors need it); otherwise it returns as soon as the
// kernels are queued and its diagnostics are checked when its workspace slot
// is reused. `zero_fill` (optional) is a buffer the call zeroes on a helper
// stream while the step merge runs; later work on `stream` sees the zeros.
struct DecodeControl {
    bool synchronize = true;
    float* zero_fill = nullptr;
    int64_t zero_fill_count = 0;
    // Split decode (row-sharded multi-GPU): caller-owned row lists for all
    // rows (row r at r * list_capacity entries), the row range this call
    // scans ([scan_begin, scan_end), -1 = all rows), and which halves run.
    uint64_t* lists = nullptr;
    int32_t* list_count = nullptr;
    float* list_bound = nullptr;
    int64_t scan_begin = 0;
    int64_t scan_end = -1;
    bool scan = true;
    bool merge = true;
    // Stepwise decode (host token filter): merge steps [t_begin, t_end) with
    // the beam state in merge_state and the prefixes in seq_scratch (both
    // caller-owned, kept between calls), row verdicts in row_allow [K][V].
    int t_begin = 0;
    int t_end = 1 << 30;
    float* merge_state = nullptr;
    int32_t* seq_scratch = nullptr;
    const uint8_t* row_allow = nullptr;
    bool force_seq = false;
    bool weights = true;
    // 16-bit log-probs read natively (d_x is then unused)
    const uint16_t* x16 = nullptr;
    bool x16_bf16 = false;
};

// Host token filter of the reference's advanced constraints
// (DBSAdvancedConstraintsC.token_filter): non-zero allows `token` after the
// beam `parent` whose tokens so far are prefix[0..prefix_len).
using TokenFilter = std::function<int(int step, int parent, const int32_t* prefix, int prefix_len, int token)>;

// Decode of one example whose candidates also pass a host token filter. The
// filter depends on each beam's prefix, so the decode runs one step at a
// time: the device scans the step's rows with the filter's verdicts and
// merges the step; the host reads the beams back and asks the filter about
// the next step's tokens, in the reference's order (parent ascending, token
// ascending, only tokens that pass the forced / banned / min-EOS / n-gram
// checks). Synchronous.
void decode_filtered(const Options& opt, const float* d_x, int V, const ExampleSpec& ex, const uint8_t* h_banned,
                     const int32_t* h_forced, const CallConstraints& cons, const Outputs& out, const Layout& layout,
                     cudaStream_t stream, DecodeStats* stats, const TokenFilter& filter);

// Source of a model-driven decode's log-probs: fills step t's [K][V] rows at
// d_rows (device) from the previous step's tokens and the final scores of the
// decode so far (the reference's DBSModelStepFn contract).
using StepRows = std::function<void(int step, const int32_t* prev_tokens, const float* prev_scores, float* d_rows)>;

// Decode of one example whose rows arrive one step at a time (the model-step
// API): each step's rows are produced after the previous step is merged, the
// device scans and merges that step, and the beams carry over in device
// memory, so the work is linear in the number of steps. d_x holds [T][K][V]
// (row (t, k) at (t * K + k) * V) and is filled by `rows`; input validation
// is the caller's (the rows exist on the host first). Synchronous.
void decode_model_steps(const Options& opt, float* d_x, int V, const ExampleSpec& ex, const Outputs& out,
                        const Layout& layout, cudaStream_t stream, DecodeStats* stats, const StepRows& rows);

// Row-list capacity C of one example (the per-row candidate list length the
// row scan keeps): N = P in pool mode else K, plus slack with sequence
// constraints, cut to the merge's per-step capacity.
int list_capacity(const Options& opt, int K, bool pool, bool dynamic);

void decode(const Options& opt, const float* d_x, int V, const std::vector<ExampleSpec>& ex,
            const CallConstraints& cons, const Outputs& out, const Layout& layout, bool pool,
            bool weights, cudaStream_t stream, DecodeStats* stats, const DecodeControl& ctl);

// Diagnostics of the most recent decode whose counters have been read back
// (process-wide): rows rescanned by the step merge, device wait timeouts,
// and rows the row scan read a second time (a speculative threshold that
// kept fewer than the row's list length).
void last_decode_diagnostics(unsigned long long* merge_rescans, unsigned long long* timeouts,
                             unsigned long long* row_rescans = nullptr);

// Kernel launches this library has queued in this process.
long long kernel_launches();

struct BackwardInputs {
    // trace (device), tight layout from `decode`
    const int32_t* parents = nullptr;
    const int32_t* tokens = nullptr;
    const int32_t* lengths = nullptr;
    const float* weights = nullptr;
    const uint8_t* from_logprob = nullptr;
    const int32_t* pool_parents = nullptr;
    const int32_t* pool_tokens = nullptr;
    const int32_t* pool_lengths = nullptr;
    const float* relaxed_weights = nullptr;
    const uint8_t* pool_from_logprob = nullptr;
    const float* grad_selected = nullptr;  // tight [T_e,K_e]
    const float* grad_relaxed = nullptr;   // tight [T_e,P_e]
    const float* grad_final = nullptr;     // [K_e]
};

struct BackwardOutputs {
    float* grad_dense = nullptr;       // tight [T_e,K_e,V], zero-filled here
    int64_t* sparse_indices = nullptr; // [sparse_total]
    float* sparse_values = nullptr;
    int64_t* sparse_counts = nullptr;  // [B]
    float* grad_initial = nullptr;     // [final_total]
};

void backward(const Options& opt, int V, const std::vector<ExampleSpec>& ex, const Layout& layout,
              const BackwardInputs& in, const BackwardOutputs& out, cudaStream_t stream,
              bool zero_dense = true);

// Sparse backward of a uniform batch (every example has T steps and the
// options' beam size) that allocates no device or pinned memory: its scratch
// is a static device array (one per device, so calls on one device must not
// overlap). Throws LengthError beyond the scratch limits.
void backward_sparse_noalloc(const Options& opt, int V, int B, int T, const BackwardInputs& in,
                             const BackwardOutputs& out, cudaStream_t stream);

int device_sm_count();

// Live kernel timing: every launch of a kernel whose bit is set in the mask is
// bracketed by a pair of CUDA events recorded on the launch stream; read()
// waits for them and returns the summed device time per kernel.
enum ProfiledKernel { kValidate = 0, kRowScan = 1, kStepMerge = 2, kWeights = 3, kFillZero = 4, kBackward = 5,
                      kProfiledKernels = 6 };
void profile_enable(unsigned mask);
void profile_reset();
void profile_read(int kernel, double* total_ms, long long* launches);

}  // namespace dbs_host
