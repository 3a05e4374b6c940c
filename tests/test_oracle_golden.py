"""Pins the CPU oracle (oracle/liboracle.so) before anything trusts it:

1. against the known-answer vectors of the reference's own unit tests
   (tests/golden/ref_kat.npz, produced by the reference's CPU backend and
   checked there against each test's expected formula);
2. against the reference's CPU backend itself (oracle/_ref), built from the
   reference sources in this container, on every seeded case of
   tests/abi_cases.py — skipped where oracle/_ref is absent.
"""
import pytest

import abi_cases
from kat_runner import HostBackend, compare, run_kat


def test_oracle_matches_reference_known_answers(oracle, golden):
    got = run_kat(HostBackend(oracle))
    bad = compare(got, golden)
    assert not bad, "\n".join(bad)


def test_reference_backend_reproduces_golden(ref_cpu, golden):
    got = run_kat(HostBackend(ref_cpu))
    assert not compare(got, golden)


@pytest.mark.parametrize("case", list(abi_cases.cases()), ids=lambda c: c[0])
def test_oracle_matches_reference_backend(case, oracle, ref_cpu):
    cid, fn, args = case
    want = abi_cases.run_case(HostBackend(ref_cpu), fn, args)
    got = abi_cases.run_case(HostBackend(oracle), fn, args)
    msgs = abi_cases.compare_outputs(got, want)
    assert not msgs, f"{cid}: " + "; ".join(msgs)
