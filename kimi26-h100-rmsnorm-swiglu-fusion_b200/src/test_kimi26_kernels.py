"""The reference's Kimi correctness script (its src/test_kimi26_kernels.py),
runnable as ``python -m src.test_kimi26_kernels`` with the same PASS lines and
closing sentence.  A thin driver over this repository's GPU parity tests: it
runs, through pytest, the reference's own check restated in
tests/test_gpu_modules.py (q_b and kv_b at 512 tokens, V1 and V3, seed 1234,
bf16, max-abs <= 3.5e-2 against linear(norm(x))) and the full-size oracle
parity of tests/test_gpu_fused.py for the same two shapes, and reports each
case."""

from __future__ import annotations

import os

_REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
_TESTS = os.path.join(_REPO, "tests")

CASES = [f"test_gpu_modules.py::test_reference_kimi_kernel_check[{v}-{c}]"
         for c in ("kimi_q_b", "kimi_kv_b") for v in ("V1", "V3")] + \
        [f"test_gpu_fused.py::test_baseline_configs_full_size[{c}]"
         for c in ("kimi_q_b", "kimi_kv_b")]


class _Outcomes:
    """pytest plugin recording each case's outcome."""

    def __init__(self):
        self.result = {}

    def pytest_runtest_logreport(self, report):
        if report.when == "call" or report.outcome != "passed":
            self.result[report.nodeid.split("/")[-1]] = report.outcome


def main() -> None:
    import pytest
    import torch

    if not torch.cuda.is_available():
        raise SystemExit("CUDA is required.")
    if not os.path.isdir(_TESTS):
        raise SystemExit(f"the parity tests are not present ({_TESTS})")
    print(f"GPU: {torch.cuda.get_device_name(0)}")
    print(f"Torch: {torch.__version__}")
    rec = _Outcomes()
    rc = pytest.main(["-q", "-p", "no:cacheprovider", "--rootdir", _REPO] +
                     [os.path.join(_TESTS, c) for c in CASES], plugins=[rec])
    for case in CASES:
        outcome = rec.result.get(case, "not run")
        print(f"{'PASS' if outcome == 'passed' else 'FAIL'}: {case} ({outcome})")
    if rc != 0 or any(rec.result.get(c) != "passed" for c in CASES):
        raise SystemExit(1)
    print("All Kimi K2.6 RMSNorm fusion kernel tests passed.")


if __name__ == "__main__":
    main()
