/*
 * Drop-in C ABI of the differentiable beam search library, served by the
 * B200 device engine (libdbs.so built from differentiable-beam-search-cuda_b200/csrc).
 *
 * Every type and function below keeps the exact layout, signature and return
 * contract of the reference interface it replaces (maged15/
 * differentiable-beam-search-cuda, include/dbs.h, ABI version 10, symbol
 * version node DBS_0.6); each declaration cites the reference line. Log-prob,
 * constraint and gradient pointers may be host or device memory: device
 * pointers are used in place, host pointers are staged. Result and backward
 * accessors always return host pointers owned by the handle.
 *
 * Return codes: 0 success, -1 null / invalid handle or output pointer,
 * -2 the call failed (message in dbs_last_error / dbs_last_global_error),
 * -3 unknown failure.
 */
#ifndef DBS_B200_DBS_H
#define DBS_B200_DBS_H

#include <stdint.h>

#if defined(__GNUC__) || defined(__clang__)
#define DBS_EXPORT __attribute__((visibility("default")))
#else
#define DBS_EXPORT
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define DBS_ABI_VERSION 10
#define DBS_VERSION_MAJOR 1
#define DBS_VERSION_MINOR 0
#define DBS_VERSION_PATCH 0

/* include/dbs.h:29-44 (64 bytes; offsets pinned by python/torch_dbs.py:20-76). */
typedef struct DBSOptionsC {
    int beam_size;
    int eos_token;
    float selected_temperature;
    float soft_topk_temperature;
    int relaxed_pool_multiplier;
    int vocab_block;
    float length_penalty_alpha;
    float soft_topk_tolerance;
    int soft_topk_max_iters;
    int min_length;
    int validate_inputs;      /* samples <= 1000 elements for NaN/+Inf */
    int64_t max_dense_gradient_elements;
    int reserved0;
    int reserved1;
} DBSOptionsC;

/* include/dbs.h:46-50 */
typedef struct DBSDecoderHandle DBSDecoderHandle;
typedef struct DBSResultHandle DBSResultHandle;
typedef struct DBSBackwardHandle DBSBackwardHandle;
typedef struct DBSBatchResultHandle DBSBatchResultHandle;
typedef struct DBSWorkspaceHandle DBSWorkspaceHandle;

/* include/dbs.h:53-62 */
typedef int (*DBSModelStepFn)(void* user_data, int batch_index, int step,
                              const int32_t* prev_tokens, const float* prev_scores,
                              int beam_size, int vocab_size, float* out_log_probs);

/* include/dbs.h:64-72. The callback is host code: with a non-null
 * token_filter, dbs_decode_constrained_ex decodes one step at a time, asks
 * the filter about each step's candidates on the host (in the reference's
 * order: parent ascending, token ascending, only tokens that pass the
 * forced / banned / minimum-length / n-gram checks) and scans and merges the
 * step on the device with its verdicts. */
typedef int (*DBSTokenFilterFn)(void* user_data, int batch_index, int step, int parent_beam,
                                const int32_t* prefix_tokens, int prefix_len, int token);

/* include/dbs.h:74-83 */
typedef struct DBSAdvancedConstraintsC {
    const uint8_t* banned_tokens;      /* [V], optional */
    const int32_t* forced_tokens;      /* [T], optional, -1 = not forced */
    int min_length;                    /* negative = decoder default */
    float repetition_penalty;          /* <=1 disables */
    int no_repeat_ngram_size;          /* <=0 disables */
    DBSTokenFilterFn token_filter;     /* optional host callback, see DBSTokenFilterFn */
    void* token_filter_user_data;
    int batch_index;
} DBSAdvancedConstraintsC;

/* include/dbs.h:85-104. last_kernel is 5 (CUDA) for every device decode. */
typedef struct DBSStatsC {
    int abi_version;
    int last_kernel;
    int used_sparse_backward;
    int used_dense_backward;
    int used_batch_threads;
    int used_model_step_callback;
    int last_error_category;           /* 0 none, 1 invalid argument, 2 runtime, 3 allocation, 4 overflow */
    int64_t last_decode_ns;
    int64_t last_backward_ns;
    int64_t last_allocation_bytes;
    int64_t last_selected_count;
    int64_t last_pool_count;
    int64_t last_logprob_count;
    int64_t last_sparse_grad_count;
    int64_t total_allocator_calls;
    int64_t total_allocator_bytes;
    int64_t reserved_stats0;
    int64_t reserved_stats1;
} DBSStatsC;

/* include/dbs.h:106-110 */
typedef enum DBSDataTypeC {
    DBS_DTYPE_F32 = 0,
    DBS_DTYPE_F16 = 1,
    DBS_DTYPE_BF16 = 2
} DBSDataTypeC;

/* Version and errors: include/dbs.h:112-114 */
DBS_EXPORT int dbs_abi_version(void);
DBS_EXPORT const char* dbs_version_string(void);
DBS_EXPORT const char* dbs_last_global_error(void);

/* Host workspace for the model-step decode: include/dbs.h:116-119 */
DBS_EXPORT int dbs_workspace_create(DBSWorkspaceHandle** out_workspace);
DBS_EXPORT void dbs_workspace_destroy(DBSWorkspaceHandle* workspace);
DBS_EXPORT int dbs_workspace_reserve(DBSWorkspaceHandle* workspace, int64_t float_count, int64_t int_count);
DBS_EXPORT int64_t dbs_workspace_allocated_bytes(DBSWorkspaceHandle* workspace);

/* Decoder lifetime: include/dbs.h:121-124 */
DBS_EXPORT int dbs_create_ex(DBSOptionsC options, DBSDecoderHandle** out_handle);
DBS_EXPORT DBSDecoderHandle* dbs_create(DBSOptionsC options);
DBS_EXPORT void dbs_destroy(DBSDecoderHandle* handle);
DBS_EXPORT const char* dbs_last_error(DBSDecoderHandle* handle);

/* [T,K,V] decode: include/dbs.h:126-132 */
DBS_EXPORT int dbs_decode(DBSDecoderHandle* handle, const float* log_probs, int steps,
                          int vocab_size, DBSResultHandle** out_result);

/* fp16 / bf16 decode (exact widening to fp32): include/dbs.h:134-152 */
DBS_EXPORT int dbs_decode_typed(DBSDecoderHandle* handle, const void* log_probs, int data_type,
                                int steps, int vocab_size, DBSResultHandle** out_result);
DBS_EXPORT int dbs_decode_batch_typed(DBSDecoderHandle* handle, const void* log_probs, int data_type,
                                      int batch_size, int steps, int vocab_size, int num_threads,
                                      DBSBatchResultHandle** out_result);

/* Constrained decode: include/dbs.h:154-172 */
DBS_EXPORT int dbs_decode_constrained(DBSDecoderHandle* handle, const float* log_probs, int steps,
                                      int vocab_size, const uint8_t* banned_tokens,
                                      const int32_t* forced_tokens, int min_length,
                                      DBSResultHandle** out_result);
DBS_EXPORT int dbs_decode_constrained_ex(DBSDecoderHandle* handle, const float* log_probs, int steps,
                                         int vocab_size, const DBSAdvancedConstraintsC* constraints,
                                         DBSResultHandle** out_result);

/* Model-step callback decode: include/dbs.h:174-193 */
DBS_EXPORT int dbs_decode_model_steps(DBSDecoderHandle* handle, DBSModelStepFn step_fn, void* user_data,
                                      int batch_index, int steps, int vocab_size,
                                      DBSResultHandle** out_result);
DBS_EXPORT int dbs_decode_model_steps_with_workspace(DBSDecoderHandle* handle, DBSWorkspaceHandle* workspace,
                                                     DBSModelStepFn step_fn, void* user_data,
                                                     int batch_index, int steps, int vocab_size,
                                                     DBSResultHandle** out_result);

/* Batched decode: include/dbs.h:195-220. num_threads is accepted for
 * compatibility; the whole batch runs as one set of device launches. */
DBS_EXPORT int dbs_decode_batch(DBSDecoderHandle* handle, const float* log_probs, int batch_size,
                                int steps, int vocab_size, int num_threads,
                                DBSBatchResultHandle** out_result);
DBS_EXPORT int dbs_decode_batch_variable(DBSDecoderHandle* handle, const float* log_probs, int batch_size,
                                         int max_steps, int max_beam_size, int vocab_size,
                                         const int32_t* steps_per_example,
                                         const int32_t* beam_sizes_per_example,
                                         const int32_t* eos_tokens_per_example,
                                         const int32_t* min_lengths_per_example,
                                         const uint8_t* banned_tokens_per_example,
                                         const int32_t* forced_tokens_per_example, int num_threads,
                                         DBSBatchResultHandle** out_result);

/* Surrogate backward: include/dbs.h:222-256 (dbs_backward and
 * dbs_backward_default are the sparse backward). */
DBS_EXPORT int dbs_backward(DBSDecoderHandle* handle, const DBSResultHandle* result,
                            const float* grad_selected_weights, const float* grad_relaxed_weights,
                            const float* grad_final_scores, DBSBackwardHandle** out_backward);
DBS_EXPORT int dbs_backward_dense(DBSDecoderHandle* handle, const DBSResultHandle* result,
                                  const float* grad_selected_weights, const float* grad_relaxed_weights,
                                  const float* grad_final_scores, DBSBackwardHandle** out_backward);
DBS_EXPORT int dbs_backward_sparse(DBSDecoderHandle* handle, const DBSResultHandle* result,
                                   const float* grad_selected_weights, const float* grad_relaxed_weights,
                                   const float* grad_final_scores, DBSBackwardHandle** out_backward);
DBS_EXPORT int dbs_backward_default(DBSDecoderHandle* handle, const DBSResultHandle* result,
                                    const float* grad_selected_weights, const float* grad_relaxed_weights,
                                    const float* grad_final_scores, DBSBackwardHandle** out_backward);

/* Release: include/dbs.h:258-260 */
DBS_EXPORT void dbs_free_result(DBSResultHandle* result);
DBS_EXPORT void dbs_free_batch_result(DBSBatchResultHandle* result);
DBS_EXPORT void dbs_free_backward(DBSBackwardHandle* result);

/* Batch access: include/dbs.h:262-263 (borrowed pointer). */
DBS_EXPORT int dbs_batch_result_size(const DBSBatchResultHandle* result);
DBS_EXPORT const DBSResultHandle* dbs_batch_result_at(const DBSBatchResultHandle* result, int batch_index);

/* Result accessors: include/dbs.h:265-284 */
DBS_EXPORT int dbs_result_steps(const DBSResultHandle* result);
DBS_EXPORT int dbs_result_beam_size(const DBSResultHandle* result);
DBS_EXPORT int dbs_result_vocab_size(const DBSResultHandle* result);
DBS_EXPORT int dbs_result_pool_size(const DBSResultHandle* result);
DBS_EXPORT const int32_t* dbs_result_tokens(const DBSResultHandle* result);
DBS_EXPORT const int32_t* dbs_result_parents(const DBSResultHandle* result);
DBS_EXPORT const int32_t* dbs_result_lengths(const DBSResultHandle* result);
DBS_EXPORT const float* dbs_result_scores(const DBSResultHandle* result);
DBS_EXPORT const float* dbs_result_raw_scores(const DBSResultHandle* result);
DBS_EXPORT const float* dbs_result_weights(const DBSResultHandle* result);
DBS_EXPORT const float* dbs_result_final_scores(const DBSResultHandle* result);
DBS_EXPORT const float* dbs_result_final_raw_scores(const DBSResultHandle* result);
DBS_EXPORT const float* dbs_result_relaxed_weights(const DBSResultHandle* result);
DBS_EXPORT const int32_t* dbs_result_pool_tokens(const DBSResultHandle* result);
DBS_EXPORT const int32_t* dbs_result_pool_parents(const DBSResultHandle* result);
DBS_EXPORT const int32_t* dbs_result_pool_lengths(const DBSResultHandle* result);
DBS_EXPORT const float* dbs_result_pool_scores(const DBSResultHandle* result);
DBS_EXPORT const float* dbs_result_pool_raw_scores(const DBSResultHandle* result);

/* Backward accessors: include/dbs.h:286-291 */
DBS_EXPORT const float* dbs_backward_grad_log_probs(const DBSBackwardHandle* result);
DBS_EXPORT const float* dbs_backward_grad_initial_scores(const DBSBackwardHandle* result);
DBS_EXPORT const int64_t* dbs_backward_sparse_logprob_indices(const DBSBackwardHandle* result);
DBS_EXPORT const float* dbs_backward_sparse_logprob_values(const DBSBackwardHandle* result);
DBS_EXPORT int64_t dbs_backward_sparse_logprob_count(const DBSBackwardHandle* result);
DBS_EXPORT int dbs_backward_is_sparse(const DBSBackwardHandle* result);

/* Counts: include/dbs.h:293-297 */
DBS_EXPORT int64_t dbs_result_selected_count(const DBSResultHandle* result);
DBS_EXPORT int64_t dbs_result_pool_count(const DBSResultHandle* result);
DBS_EXPORT int64_t dbs_result_logprob_count(const DBSResultHandle* result);
DBS_EXPORT int64_t dbs_backward_grad_log_probs_count(const DBSResultHandle* result);
DBS_EXPORT int64_t dbs_backward_grad_initial_scores_count(const DBSResultHandle* result);

/* Result utilities: include/dbs.h:299-302 (the manifest validator is a
 * deprecated stub that always fails). */
DBS_EXPORT int64_t dbs_result_eos_count(const DBSResultHandle* result, int eos_token);
DBS_EXPORT int dbs_result_validate_deterministic_order(const DBSResultHandle* result);
DBS_EXPORT int dbs_result_summary_json(const DBSResultHandle* result, int eos_token, char* out_json,
                                       int64_t out_json_capacity);
DBS_EXPORT int dbs_validate_production_gate_manifest(const char* manifest_json, char* out_error,
                                                     int64_t out_error_capacity);

/* Host capability and observability: include/dbs.h:304-317 */
DBS_EXPORT int dbs_has_avx512(void);
DBS_EXPORT int dbs_has_avx2(void);
DBS_EXPORT int dbs_has_sse42(void);
DBS_EXPORT int dbs_has_neon(void);
DBS_EXPORT const char* dbs_selected_kernel_name(void);
DBS_EXPORT int dbs_get_stats(DBSDecoderHandle* handle, DBSStatsC* out_stats);
DBS_EXPORT int dbs_get_stats_json(DBSDecoderHandle* handle, char* out_json, int64_t out_json_capacity);
DBS_EXPORT int dbs_is_deterministic(void);
DBS_EXPORT int dbs_set_deterministic_seed(DBSDecoderHandle* handle, uint64_t seed);
DBS_EXPORT uint64_t dbs_get_deterministic_seed(DBSDecoderHandle* handle);
DBS_EXPORT void dbs_allocator_counters_reset(void);
DBS_EXPORT int64_t dbs_allocator_call_count(void);
DBS_EXPORT int64_t dbs_allocator_byte_count(void);
DBS_EXPORT void dbs_reset_stats(DBSDecoderHandle* handle);

#ifdef __cplusplus
}
#endif

#endif /* DBS_B200_DBS_H */
