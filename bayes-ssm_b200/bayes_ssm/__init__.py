"""B200-native (sm_100a) drop-in for catid/bayes-ssm's dense Bayesian layers.

Same public surface as the reference package ``bayes_ssm/__init__.py:2-20``.
CUDA work runs in hand-written kernels behind a C ABI (``lib/libbayes_ssm_b200.so``,
declared in ``include/bayes_ssm_b200.h``).
"""
from .bayesian_layer import (
    BayesianLayer,
    bayesian_layer,
    make_diagonal_dynamics,
    make_rotation_dynamics,
    make_rotation_process_covariances,
)
from .replay_ssm import (
    ReplaySSM,
    associative_static_bayesian,
    associative_static_bayesian_cuda,
)

__all__ = [
    "BayesianLayer", "bayesian_layer", "make_diagonal_dynamics",
    "make_rotation_dynamics", "make_rotation_process_covariances",
    "ReplaySSM", "associative_static_bayesian",
    "associative_static_bayesian_cuda",
]
