"""The reference's own known-answer tests (mimi-rs/tests/cuda_tests.rs and
tests/tensor_tests.rs, restated in tests/golden/known_answers.json), run
through the GPU kernels."""
import pytest

from known_answers import GpuRunner, load_cases, run_case

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", load_cases(), ids=lambda c: c["name"])
def test_known_answer_gpu(xn, cuda, case):
    run_case(case, GpuRunner(xn, cuda))
