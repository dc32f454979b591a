"""The oracle against the reference's own golden vectors (CPU).

Every case comes from mlirpass's fixtures (tests/fixtures/*.in.mlir and
*.generic.mlir, harvested by tests/golden/make_golden.py): a hot-path fold
op whose operands are constants, and mlir-opt 23.1.5's folded constant, or
the op left in place when the reference refuses to fold.
"""
import pytest

from golden_cases import case_id, check_case, element_cases, load_cases

CASES = element_cases()


def test_vectors_present():
    cases = load_cases()
    assert len(cases) >= 50
    ops = {c["op"] for c in cases}
    for must in ("arith.truncf", "arith.fptosi", "arith.sitofp", "arith.shli", "arith.remsi", "arith.addf",
                 "arith.divf", "arith.cmpi", "tosa.reciprocal"):
        assert must in ops
    # The reference refuses some folds: those vectors must be present too.
    assert any(c["expected"]["status"] == "not_folded" for c in cases)


@pytest.mark.parametrize("case", CASES, ids=[case_id(c) for c in CASES])
def test_oracle_matches_golden(case, oracle):
    check_case(case, oracle)
