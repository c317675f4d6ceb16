// Device engine for differentiable beam search on sm_100a.
//
// The decode of one example is split into three launches:
//
//   1. row scan   (dbs_row_scan_kernel)   -- every [V] log-prob row of every
//      step is streamed from HBM exactly once, fully in parallel, and reduced
//      to its best C entries by (lp desc, token asc) plus an upper bound on
//      everything it dropped. Beam state is not needed for this: for a fixed
//      parent, raw = parent + lp and rank = raw / gnmt(len+1) are monotone in
//      lp, so every candidate that can win a step comes from the head of its
//      row.
//   2. step merge (dbs_step_merge_kernel) -- one CTA per example walks the T
//      steps sequentially, merges the K row lists (plus EOS carries) under the
//      reference's six-key candidate order, proves per row that nothing the
//      scan dropped could have entered the top-N (rescanning the row from HBM
//      when it cannot), and writes backpointers, tokens, lengths, scores and
//      the relaxed pool.
//   3. weights    (dbs_weights_kernel)    -- selected softmax and the
//      sigmoid-bisection relaxed pool weights, one warp per (example, step).
//
// The sparse / dense surrogate backward is a per-example reverse sweep over
// the trace (dbs_backward_kernel).
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

namespace dbs_dev {

// Static (beam-state independent) per-example decode parameters. Log-prob
// row (t, k) of example e starts at element
//   x_offset + (t * k_stride + k) * V
// which covers both the uniform [B,T,K,V] layout (k_stride = K) and the
// variable-batch [B,maxT,maxK,V] layout (k_stride = maxK).
struct ExampleDesc {
    int64_t x_offset;        // element offset of (t=0, k=0, v=0)
    int64_t row_begin;       // first global row index of this example
    int64_t list_offset;     // first list entry (u64) of this example
    int64_t sel_offset;      // offset of [T,K] outputs (elements)
    int64_t pool_offset;     // offset of [T,P] outputs (elements)
    int64_t final_offset;    // offset of [K] outputs (elements)
    int64_t grad_offset;     // offset of [T,K,V] dense gradient (elements)
    int64_t sparse_offset;   // offset of [T*(K+P)] sparse entries
    int32_t T;
    int32_t K;
    int32_t k_stride;        // rows per step in the input layout
    int32_t P;               // relaxed pool size (output width of the pool)
    int32_t N;               // candidates selected per step (P or K)
    int32_t C;               // row list capacity (at most N; shorter lists are proven per step)
    int32_t ext0;            // extra entries of beam 0's rows (compact merge only): a step's lists
                             // are K rows of C entries, then beam 0's entries C .. C + ext0 - 1
    int32_t sel_stride;      // K-dimension stride of [T,K] outputs
    int32_t pool_stride;     // P-dimension stride of [T,P] outputs
    int32_t sel_t_stride;    // T-dimension stride (elements) of selected outputs
    int32_t pool_t_stride;   // T-dimension stride (elements) of pool outputs
    int32_t eos;
    int32_t min_length;      // effective min length for EOS
    const uint8_t* banned;   // [V] or nullptr
    const int32_t* forced;   // [>=T] or nullptr
};

// Options shared by every example of one call.
struct DecodeParams {
    const float* x;
    // 16-bit log-probs read natively instead of x (fp16 or bf16 bit
    // patterns, widened exactly on load); nullptr for fp32 inputs
    const uint16_t* x16;
    int32_t x16_bf16;
    int32_t V;
    int32_t B;
    int64_t total_rows;
    const ExampleDesc* desc;      // [B] (device)
    const int64_t* row_prefix;    // [B+1] (device) global row index per example
    const float* pen;             // [Lmax+1] gnmt(l) for l>=1, pen[0]=pen[1]
    const float* inv_pen;         // [Lmax+1] 1.0f / pen[l]
    int32_t Lmax;
    float selected_temperature;
    float soft_topk_temperature;
    float soft_topk_tolerance;
    int32_t soft_topk_max_iters;
    float repetition_penalty;     // > 1 enables
    float log_repetition_penalty; // logf(repetition_penalty), host computed
    int32_t no_repeat_ngram;      // > 0 enables
    int32_t validate_inputs;
    // Stepwise decoding (host token filters): the merge runs steps
    // [t_begin, t_end) only, loading the beam state from merge_state when
    // t_begin > 0 and storing it there when steps remain; row_allow [K][V]
    // holds the host filter's verdict for the rows scanned in this launch;
    // force_seq keeps the beams' token prefixes without sequence constraints.
    int32_t t_begin;
    int32_t t_end;
    float* merge_state;            // [B][4][max K]: raw, len, ended, prefix length
    const uint8_t* row_allow;
    int32_t force_seq;
    // Short row lists (many-example relaxed-pool decodes): the one live row
    // of step 0, (t=0, k=0), gets a list of up to min(N, K*C, 1024) entries in the
    // list space of step 0's K rows (the other K-1 rows of step 0 are never
    // extended). The main row scan skips that row; a second launch with
    // first_rows_only = 1 scans exactly those rows (claim i -> row_prefix[i]);
    // the step merge reads step 0 as that one list.
    int32_t first_row_apart;
    int32_t first_rows_only;
    // Step-major row claims of the fused decode (a uniform batch of B
    // examples, K beams, row stride step_major_tk = T*K per example): with
    // step_major_bk = B*K, claim c scans step c / (B*K) of example
    // (c / K) % B, beam c % K, so the rows of early steps are listed first.
    // (The separate row-scan launches claim rows in order.)
    int64_t step_major_bk;
    int64_t step_major_tk;
    // workspace
    uint64_t* lists;              // row lists, key = ord(lp)<<32 | ~token
    int32_t* list_count;          // [total_rows]
    float* list_bound;            // [total_rows] max dropped lp (-inf: none)
    int32_t* status;              // [B] 0 ok, 1 NaN/+Inf sampled
    unsigned long long* counters; // [4]: row-scan second passes, merge rescans, next row claim, wait timeouts
    int32_t* seq_scratch;         // [B, 2, K, T] beam prefixes (constraints only)
    // outputs (element pointers; any may be null except the trace needed by
    // later stages)
    int32_t* parents;
    int32_t* tokens;
    int32_t* lengths;
    float* raw_scores;
    float* scores;
    float* weights;
    uint8_t* from_logprob;
    int32_t* pool_parents;
    int32_t* pool_tokens;
    int32_t* pool_lengths;
    float* pool_raw_scores;
    float* pool_scores;
    float* relaxed_weights;
    uint8_t* pool_from_logprob;
    float* final_raw_scores;
    float* final_scores;
};

struct BackwardParams {
    int32_t V;
    int32_t B;
    int32_t max_T;                // row stride of step_counts
    const ExampleDesc* desc;
    const float* inv_pen;
    int32_t Lmax;
    float selected_temperature;
    float soft_topk_temperature;
    // trace (same layout as DecodeParams outputs)
    const int32_t* parents;
    const int32_t* tokens;
    const int32_t* lengths;
    const float* weights;
    const uint8_t* from_logprob;
    const int32_t* pool_parents;
    const int32_t* pool_tokens;
    const int32_t* pool_lengths;
    const float* relaxed_weights;
    const uint8_t* pool_from_logprob;
    // gradient inputs (null = absent); same offsets as the trace outputs
    const float* grad_selected;
    const float* grad_relaxed;
    const float* grad_final;
    // outputs
    float* grad_dense;            // [.., T,K,V] at desc.grad_offset, pre-zeroed
    int64_t* sparse_indices;      // [.., T*(K+P)] at desc.sparse_offset
    float* sparse_values;
    int64_t* sparse_counts;       // [B]
    int32_t* step_counts;         // [B, T] scratch
    float* grad_initial;          // [B, K] at desc.final_offset
};

// Host-side launchers (dbs_kernels.cu). All are asynchronous on `stream`.
cudaError_t launch_validate(const DecodeParams& p, cudaStream_t stream);
// Scans the rows claimed from counters[2] (the first row to scan) up to
// p.total_rows; `rows` is how many that is (-1: p.total_rows), for sizing.
// speculate: -1 decides by the rows per warp, 1 forces speculative thresholds
// for long lists (a launch seeded from an earlier one's spec_seed).
cudaError_t launch_row_scan(const DecodeParams& p, int max_C, int num_sms, cudaStream_t stream, int64_t rows = -1,
                            int speculate = -1);
// max_threads caps the CTA size of the selection merge (256 lets two merge
// CTAs share an SM).
cudaError_t launch_step_merge(const DecodeParams& p, int max_K, int max_C, int max_T,
                              int max_N, bool need_sequences, cudaStream_t stream, int max_threads = 0,
                              int max_ext = 0);
// Whether launch_step_merge runs the compact merge for these sizes, with
// beam 0's lists max_ext entries longer (only the compact merge reads
// ExampleDesc::ext0, so the engine sets it only when this holds).
bool compact_merge_applies(int max_K, int max_C, int max_ext, int max_N, bool need_sequences,
                           bool first_row_apart);
// Kernel launches made by this library in this process (every launcher
// counts the launches it queues).
long long kernel_launch_count();
cudaError_t launch_weights(const DecodeParams& p, int max_T, int max_K, int max_P,
                           cudaStream_t stream);
// Fused decode of a uniform batch without sequence constraints (rows
// claimed step-major; p.merge_state holds [B][4][max_K] beams when
// merge_ctas < B; step_done [B*T] zeroed). cudaErrorNotSupported when the
// shape or the device does not allow it (the caller then scans and merges
// in separate launches).
cudaError_t launch_fused_decode(const DecodeParams& p, int max_K, int max_C, int max_ext, int max_N,
                                int merge_ctas, unsigned int* step_done, int num_sms, cudaStream_t stream);
cudaError_t launch_backward(const BackwardParams& p, int max_K, int max_P, bool sparse,
                            cudaStream_t stream);
// blocks_per_sm: 4 fills the GPU; 1 leaves three quarters of every SM's
// registers and thread slots to a kernel running beside the fill (the merge).
cudaError_t launch_fill_zero(float* dst, int64_t count, int num_sms, cudaStream_t stream, int blocks_per_sm = 4);
// Same result through bulk (TMA) stores from one 32-thread CTA per SM; leaves
// the SMs' load/store pipes and registers to a kernel running beside it.
cudaError_t launch_fill_zero_bulk(float* dst, int64_t count, int num_sms, cudaStream_t stream);

// Sparse backward of a uniform batch whose only scratch is a static device
// array (no allocation on the call path); inv_pen_host holds 1/gnmt(l) for
// l = 0 .. T+1. Returns cudaErrorInvalidValue beyond the limits below.
constexpr int kNoAllocMaxSteps = 510;
constexpr int kNoAllocMaxStepCounts = 1 << 18;   // batch_size * steps (1 MiB of int32)
constexpr int kNoAllocMaxBeamPlusPool = 4096;
cudaError_t launch_backward_noalloc(const BackwardParams& p, int T, int K, int P, const float* inv_pen_host,
                                    cudaStream_t stream);
// Looks up this device's scratch address and sets the kernel's shared-memory
// limit; the first call on each device does this work.
cudaError_t noalloc_prepare();

// Limits of this implementation.
constexpr int kMaxMergeCandidates = 8192;   // K * C per step handled by one CTA
// Longest list of the step-0 row of a short-list decode (a shorter list than
// the pool only costs a rescan; longer ones would not fit the scan's shared
// memory for every pool size).
constexpr int kStep0ListMax = 1024;
constexpr int kMergeThreads = 512;
// Compact merge (no sequence constraints): CTA size and candidates per step.
constexpr int kListMergeThreads = 512;
constexpr int kListMergeMaxCandidates = 8 * kListMergeThreads;
// Fused decode (scan and merge in one cooperative launch): CTA size.
constexpr int kFusedThreads = 512;
// Speculative row-scan thresholds a warp remembers, one per list length
// (rows of one call can have different list lengths, e.g. per-example beam
// sizes); also the entries of DecodeParams::spec_seed.
constexpr int kSpecSlots = 4;

}  // namespace dbs_dev
