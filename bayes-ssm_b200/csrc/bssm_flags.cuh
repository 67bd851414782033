// bssm_flags.cuh -- the value-check flags of one element, shared by the check
// kernel and the kernels that compute the checks of what they write.
//
// bayesian_layer validates its inputs before any recurrence runs
// (catid/bayes-ssm bayes_ssm/bayesian_layer.py:105-128): every tensor finite,
// process variances nonnegative, observation variances strictly positive.
#pragma once

#include "bayes_ssm_b200.h"

namespace bssm {

__device__ __forceinline__ unsigned check_flags_of(float v) {
    unsigned f = 0;
    if (!isfinite(v)) f |= BSSM_CHECK_NONFINITE;
    if (v <= 0.f) f |= BSSM_CHECK_NOT_POSITIVE;  // NaN compares false: it only sets the first flag
    if (v < 0.f) f |= BSSM_CHECK_NEGATIVE;
    return f;
}

}  // namespace bssm
