/*
 * CPU oracle for the differentiable beam search hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker the parity tests and
 * the CPU baseline arm of bench.py compare against; the product never links,
 * loads or calls it.
 *
 * It restates, in plain C, the reference decoder's scalar semantics
 * (maged15/differentiable-beam-search-cuda, src/differentiable_beam.cpp):
 * option defaults, sampled input validation, the per-step candidate scan with
 * constraints, top-P selection under the six-key candidate order, the
 * sigmoid-bisection relaxed pool weights, the selected softmax, finalisation,
 * and the sparse / dense surrogate backward. Parity of this restatement is
 * pinned against the reference library compiled from its own source
 * (oracle/_ref/libdbs_ref.so) and against the fixtures in tests/golden/.
 */
#ifndef DBS_ORACLE_H
#define DBS_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Options after the reference's C-ABI default substitution
 * (from_c_options, src/differentiable_beam.cpp:3145-3177). */
typedef struct oracle_options {
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
    int validate_inputs;
    int64_t max_dense_gradient_elements;
} oracle_options;

/* Decode constraints (DecodeConstraints, src/differentiable_beam.cpp:184-200).
 * min_length < 0 means "use options.min_length". */
typedef int (*oracle_token_filter)(void* user_data, int batch_index, int step, int parent_beam,
                                   const int32_t* prefix_tokens, int prefix_len, int token);

typedef struct oracle_constraints {
    const uint8_t* banned_tokens;   /* [V] or NULL */
    const int32_t* forced_tokens;   /* [T] or NULL, -1 = free */
    int min_length;
    float repetition_penalty;       /* <= 1 disables */
    int no_repeat_ngram_size;       /* <= 0 disables */
    oracle_token_filter token_filter; /* NULL or non-zero = allow (token_allowed_by_advanced_constraints, :339-349) */
    void* token_filter_user_data;
    int batch_index;
} oracle_constraints;

/* Output arrays of one decode (DecodeResult, :202-237). All are caller-owned.
 * K = beam_size, P = max(K, K * relaxed_pool_multiplier). */
typedef struct oracle_result {
    int32_t* parents;        /* [T*K] */
    int32_t* tokens;         /* [T*K] */
    int32_t* lengths;        /* [T*K] */
    float* raw_scores;       /* [T*K] */
    float* scores;           /* [T*K] */
    float* weights;          /* [T*K] */
    uint8_t* from_logprob;   /* [T*K] */
    int32_t* pool_parents;   /* [T*P] */
    int32_t* pool_tokens;    /* [T*P] */
    int32_t* pool_lengths;   /* [T*P] */
    float* pool_raw_scores;  /* [T*P] */
    float* pool_scores;      /* [T*P] */
    float* relaxed_weights;  /* [T*P] */
    uint8_t* pool_from_logprob; /* [T*P] */
    float* final_raw_scores; /* [K] */
    float* final_scores;     /* [K] */
} oracle_result;

/* Apply the C-ABI default rules to raw option fields. */
void oracle_options_from_c(int beam_size, int eos_token, float selected_temperature,
                           float soft_topk_temperature, int relaxed_pool_multiplier,
                           int vocab_block, float length_penalty_alpha,
                           float soft_topk_tolerance, int soft_topk_max_iters,
                           int min_length, int validate_inputs,
                           int64_t max_dense_gradient_elements, oracle_options* out);

int oracle_pool_size(const oracle_options* opt);

/* Returns 0 on success; non-zero with a message in oracle_last_error() for the
 * cases where the reference throws std::invalid_argument / overflow_error. */
int oracle_decode(const oracle_options* opt, const float* log_probs, int steps,
                  int vocab_size, const oracle_constraints* constraints,
                  oracle_result* out);

/* Sparse surrogate backward (backward_sparse, :1736-1791). Writes at most
 * T*(K+P) sorted unique entries; *nnz receives the count. Any of the three
 * gradient inputs may be NULL. */
int oracle_backward_sparse(const oracle_options* opt, int steps, int vocab_size,
                           const oracle_result* fwd, const float* grad_selected,
                           const float* grad_relaxed, const float* grad_final,
                           int64_t* out_indices, float* out_values, int64_t* nnz,
                           float* grad_initial);

/* Dense surrogate backward (backward, :1674-1734) into [T*K*V]. */
int oracle_backward_dense(const oracle_options* opt, int steps, int vocab_size,
                          const oracle_result* fwd, const float* grad_selected,
                          const float* grad_relaxed, const float* grad_final,
                          float* grad_log_probs, float* grad_initial);

const char* oracle_last_error(void);

#ifdef __cplusplus
}
#endif

#endif
