/*
 * Prints the layout of the C ABI's public types for whichever dbs.h is on the
 * include path: the size of each struct, the offset and size of every field,
 * the data-type enum's values, the version macros and the callback pointer
 * sizes.
 *
 * TEST INFRASTRUCTURE ONLY: oracle/Makefile compiles it once against this
 * repository's include/dbs.h and once against the reference's, and
 * tests/test_cpu_abi.py requires the two outputs to be identical (a caller
 * compiled against either header passes structs by value and by pointer).
 */
#include <stddef.h>
#include <stdio.h>

#include "dbs.h"

#define STRUCT(S) printf(#S " size %zu\n", sizeof(S))
#define FIELD(S, f) printf(#S "." #f " offset %zu size %zu\n", offsetof(S, f), sizeof(((S*)0)->f))

int main(void) {
    STRUCT(DBSOptionsC);
    FIELD(DBSOptionsC, beam_size);
    FIELD(DBSOptionsC, eos_token);
    FIELD(DBSOptionsC, selected_temperature);
    FIELD(DBSOptionsC, soft_topk_temperature);
    FIELD(DBSOptionsC, relaxed_pool_multiplier);
    FIELD(DBSOptionsC, vocab_block);
    FIELD(DBSOptionsC, length_penalty_alpha);
    FIELD(DBSOptionsC, soft_topk_tolerance);
    FIELD(DBSOptionsC, soft_topk_max_iters);
    FIELD(DBSOptionsC, min_length);
    FIELD(DBSOptionsC, validate_inputs);
    FIELD(DBSOptionsC, max_dense_gradient_elements);
    FIELD(DBSOptionsC, reserved0);
    FIELD(DBSOptionsC, reserved1);

    STRUCT(DBSAdvancedConstraintsC);
    FIELD(DBSAdvancedConstraintsC, banned_tokens);
    FIELD(DBSAdvancedConstraintsC, forced_tokens);
    FIELD(DBSAdvancedConstraintsC, min_length);
    FIELD(DBSAdvancedConstraintsC, repetition_penalty);
    FIELD(DBSAdvancedConstraintsC, no_repeat_ngram_size);
    FIELD(DBSAdvancedConstraintsC, token_filter);
    FIELD(DBSAdvancedConstraintsC, token_filter_user_data);
    FIELD(DBSAdvancedConstraintsC, batch_index);

    STRUCT(DBSStatsC);
    FIELD(DBSStatsC, abi_version);
    FIELD(DBSStatsC, last_kernel);
    FIELD(DBSStatsC, used_sparse_backward);
    FIELD(DBSStatsC, used_dense_backward);
    FIELD(DBSStatsC, used_batch_threads);
    FIELD(DBSStatsC, used_model_step_callback);
    FIELD(DBSStatsC, last_error_category);
    FIELD(DBSStatsC, last_decode_ns);
    FIELD(DBSStatsC, last_backward_ns);
    FIELD(DBSStatsC, last_allocation_bytes);
    FIELD(DBSStatsC, last_selected_count);
    FIELD(DBSStatsC, last_pool_count);
    FIELD(DBSStatsC, last_logprob_count);
    FIELD(DBSStatsC, last_sparse_grad_count);
    FIELD(DBSStatsC, total_allocator_calls);
    FIELD(DBSStatsC, total_allocator_bytes);
    FIELD(DBSStatsC, reserved_stats0);
    FIELD(DBSStatsC, reserved_stats1);

    printf("DBSDataTypeC size %zu values %d %d %d\n", sizeof(DBSDataTypeC), (int)DBS_DTYPE_F32,
           (int)DBS_DTYPE_F16, (int)DBS_DTYPE_BF16);
    printf("DBSModelStepFn size %zu DBSTokenFilterFn size %zu\n", sizeof(DBSModelStepFn),
           sizeof(DBSTokenFilterFn));
    printf("DBS_ABI_VERSION %d DBS_VERSION %d.%d.%d\n", DBS_ABI_VERSION, DBS_VERSION_MAJOR, DBS_VERSION_MINOR,
           DBS_VERSION_PATCH);
    return 0;
}
