/*
 * Device-resident extension of the dbs C ABI (not part of the reference's
 * ABI version 10; added beside it without changing any existing symbol).
 *
 * The reference interface takes host arrays and returns host-owned results
 * (include/dbs.h:126-256 of maged15/differentiable-beam-search-cuda). These
 * entry points take DEVICE pointers and a cudaStream_t (passed as void*), run
 * the whole decode / backward as stream-ordered kernel launches, and write
 * results straight into caller-owned device buffers. They are what the
 * PyTorch final_scores autograd Function (the reference's
 * python/torch_dbs_extension.py:233-303) and bench.py call.
 *
 * Output layout ("tight"): example b's [T_b, K_b] selected arrays start at
 * sum_{c<b} T_c*K_c, its [T_b, P_b] pool arrays at sum_{c<b} T_c*P_b and its
 * [K_b] final arrays at sum_{c<b} K_c, with P_b = max(K_b, K_b *
 * relaxed_pool_multiplier). For the uniform batch this is plain [B,T,K],
 * [B,T,P] and [B,K].
 */
#ifndef DBS_B200_DBS_DEVICE_H
#define DBS_B200_DBS_DEVICE_H

#include "dbs.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Device output arrays of one decode call. parents, tokens, lengths and
 * from_logprob are required. When pool_scores is NULL only the top beam_size
 * candidates of every step are selected and no pool / relaxed weights are
 * produced (the selected arrays and final scores are unchanged by this: they
 * are the head of the top-P pool). weights (selected softmax) is produced
 * only when non-NULL; relaxed_weights only with pool_scores. */
typedef struct DBSDeviceDecodeOutputs {
    int32_t* parents;
    int32_t* tokens;
    int32_t* lengths;
    uint8_t* from_logprob;
    float* raw_scores;
    float* scores;
    float* weights;
    int32_t* pool_parents;
    int32_t* pool_tokens;
    int32_t* pool_lengths;
    uint8_t* pool_from_logprob;
    float* pool_raw_scores;
    float* pool_scores;
    float* relaxed_weights;
    float* final_raw_scores;
    float* final_scores;
} DBSDeviceDecodeOutputs;

/* Uniform batch decode of device log_probs [B,T,K,V] (K = beam_size).
 * Replaces dbs_decode_batch (reference include/dbs.h:195-203) for device
 * data. With validate_inputs on, the call waits for the stream and fails with
 * -2 "log_probs contains NaN or +Inf" like the reference; otherwise it
 * returns without synchronising. */
DBS_EXPORT int dbs_device_decode_batch(DBSDecoderHandle* handle, const float* log_probs, int batch_size,
                                       int steps, int vocab_size, const DBSDeviceDecodeOutputs* outputs,
                                       void* cuda_stream);

/* Variable-length constrained batch decode of device log_probs
 * [B, max_steps, max_beam_size, V]: the per-example options of
 * dbs_decode_batch_variable (reference include/dbs.h:205-220) plus the
 * repetition penalty and no-repeat n-gram of dbs_decode_constrained_ex
 * (include/dbs.h:165-172, :74-83), which the reference's variable API cannot
 * take. steps / beams / eos / min_lengths are HOST arrays [B] (NULL = handle
 * default), banned [B,V] and forced [B,max_steps] are DEVICE arrays (NULL =
 * none). Outputs use the tight layout. */
DBS_EXPORT int dbs_device_decode_batch_variable_ex(
    DBSDecoderHandle* handle, const float* log_probs, int batch_size, int max_steps, int max_beam_size,
    int vocab_size, const int32_t* steps_per_example, const int32_t* beam_sizes_per_example,
    const int32_t* eos_tokens_per_example, const int32_t* min_lengths_per_example,
    const uint8_t* banned_tokens_per_example, const int32_t* forced_tokens_per_example,
    float repetition_penalty, int no_repeat_ngram_size, const DBSDeviceDecodeOutputs* outputs,
    void* cuda_stream);

/* Surrogate backward of a uniform batch from its device trace (the
 * reference's dbs_backward_sparse / dbs_backward_dense, include/dbs.h:222-247,
 * batched). Gradient inputs are device arrays in the tight layout or NULL.
 * Exactly one of grad_log_probs (dense [B,T,K,V], fully overwritten) or
 * sparse_indices / sparse_values ([B, T*(K+P)] capacity, example b at
 * b*T*(K+P), indices local to the example's [T*K*V]) with sparse_counts [B]
 * must be given. grad_initial_scores [B,K] is optional. Asynchronous. */
DBS_EXPORT int dbs_device_backward_batch(DBSDecoderHandle* handle, int batch_size, int steps,
                                         int vocab_size, const DBSDeviceDecodeOutputs* trace,
                                         const float* grad_selected_weights,
                                         const float* grad_relaxed_weights,
                                         const float* grad_final_scores, float* grad_log_probs,
                                         int64_t* sparse_indices, float* sparse_values,
                                         int64_t* sparse_counts, float* grad_initial_scores,
                                         void* cuda_stream);

/* dbs_device_decode_batch plus an optional buffer to zero: `zero_fill`
 * (count elements, device) is cleared on a helper stream while the step
 * merge runs, and later work on `cuda_stream` sees the zeros. The autograd
 * path uses it for the dense gradient its backward will scatter into. */
DBS_EXPORT int dbs_device_decode_batch_ex(DBSDecoderHandle* handle, const float* log_probs, int batch_size,
                                          int steps, int vocab_size, const DBSDeviceDecodeOutputs* outputs,
                                          float* zero_fill, int64_t zero_fill_count, void* cuda_stream);

/* dbs_device_backward_batch with flags; DBS_DEVICE_GRAD_PREZEROED means the
 * dense grad_log_probs already holds zeros (e.g. from zero_fill above), so
 * only the non-zero entries are written. */
#define DBS_DEVICE_GRAD_PREZEROED 1
DBS_EXPORT int dbs_device_backward_batch_ex(DBSDecoderHandle* handle, int batch_size, int steps,
                                            int vocab_size, const DBSDeviceDecodeOutputs* trace,
                                            const float* grad_selected_weights,
                                            const float* grad_relaxed_weights,
                                            const float* grad_final_scores, float* grad_log_probs,
                                            int64_t* sparse_indices, float* sparse_values,
                                            int64_t* sparse_counts, float* grad_initial_scores, int flags,
                                            void* cuda_stream);

/* Split decode of a uniform batch for row-sharded multi-GPU runs. The decode
 * is a row scan (every [V] row reduced to its best C candidates, C from
 * dbs_device_row_list_capacity) followed by the sequential step merge.
 * dbs_device_scan_rows scans rows [row_begin, row_end) of the batch (global
 * row r = (b*steps + t)*beam_size + k) into caller-owned device arrays that
 * cover all rows: lists [rows * C] (64-bit entries), list_counts [rows],
 * list_bounds [rows]; it validates the input like dbs_device_decode_batch.
 * Once every row is present (e.g. after an all-gather of each rank's range),
 * dbs_device_merge_rows runs the merge (and weights) and writes the same
 * outputs as dbs_device_decode_batch with the same log_probs. The entry
 * format is internal; only this library's scan produces lists the merge
 * accepts. with_pool must match the outputs' pool_scores (NULL or not).
 * No counterpart in the reference (its CPU decoder has no sharding). */
DBS_EXPORT int dbs_device_row_list_capacity(DBSDecoderHandle* handle, int with_pool, int* capacity);
DBS_EXPORT int dbs_device_scan_rows(DBSDecoderHandle* handle, const float* log_probs, int batch_size, int steps,
                                    int vocab_size, int with_pool, int64_t row_begin, int64_t row_end,
                                    uint64_t* lists, int32_t* list_counts, float* list_bounds, void* cuda_stream);
DBS_EXPORT int dbs_device_merge_rows(DBSDecoderHandle* handle, const float* log_probs, int batch_size, int steps,
                                     int vocab_size, const uint64_t* lists, const int32_t* list_counts,
                                     const float* list_bounds, const DBSDeviceDecodeOutputs* outputs,
                                     void* cuda_stream);

/* Sparse backward of a uniform batch that allocates nothing on its call path:
 * same arguments, outputs and results as dbs_device_backward_batch with
 * sparse outputs (grad_log_probs NULL). For callers that must not allocate
 * device memory where they call it (a caching allocator owns the device, a
 * capture or replay region, a latency-critical loop where cudaMalloc's
 * implicit synchronisation is unacceptable). Its scratch is a static device
 * array of 1 MiB per device, which limits it to batch_size * steps <= 262144,
 * steps <= 510 and beam + pool <= 4096 (-2 with a "takes at most" message
 * beyond them). The first call on a device looks the scratch up and loads
 * the module, so make one call before any region that forbids that. The
 * scratch is shared by all calls on a device: calls must not overlap in time
 * (two streams would race); calls in a row on one stream are fine. No
 * counterpart in the reference, whose backward allocates host memory. */
DBS_EXPORT int dbs_device_backward_sparse_noalloc(DBSDecoderHandle* handle, int batch_size, int steps,
                                                  int vocab_size, const DBSDeviceDecodeOutputs* trace,
                                                  const float* grad_selected_weights,
                                                  const float* grad_relaxed_weights,
                                                  const float* grad_final_scores, int64_t* sparse_indices,
                                                  float* sparse_values, int64_t* sparse_counts,
                                                  float* grad_initial_scores, void* cuda_stream);

/* Diagnostics of the most recent device decode whose counters have been read
 * back (process-wide): rows the row scan read a second time from HBM (a
 * speculative threshold, learned from earlier rows, kept fewer entries than
 * the row's list length; the list stays exact) and rows the step merge could
 * not prove complete and rescanned from HBM. No counterpart in the reference. */
DBS_EXPORT int dbs_device_last_rescan_counts(DBSDecoderHandle* handle, int64_t* row_rescans,
                                             int64_t* merge_rescans);

/* Kernel launches this library has queued in this process so far (for
 * benchmarks counting the launches of a timed region). No counterpart in
 * the reference. */
DBS_EXPORT int dbs_device_kernel_launches(int64_t* count);

/* Live kernel timing for benchmarks: enable = 1 starts bracketing every
 * device launch with CUDA events on its stream, 0 stops, -1 clears the
 * totals. dbs_device_profile_read waits for the recorded events and returns
 * the summed device milliseconds and launch count of one kernel:
 * 0 validate, 1 row scan, 2 step merge, 3 weights, 4 zero fill, 5 backward.
 * No counterpart in the reference (its stats hold host wall-clock only,
 * src/differentiable_beam.cpp:3115-3143). */
DBS_EXPORT int dbs_device_profile(int enable);
DBS_EXPORT int dbs_device_profile_read(int kernel, double* total_ms, int64_t* launches);
/* Times only the kernels whose bit (1 << kernel id above) is set in `mask`
 * (0 stops timing), so a benchmark can time one kernel inside a timed region
 * with two events per launch of that kernel and none elsewhere. */
DBS_EXPORT int dbs_device_profile_kernels(unsigned mask);

#ifdef __cplusplus
}
#endif

#endif /* DBS_B200_DBS_DEVICE_H */
