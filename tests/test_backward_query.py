"""Constant-index (backward-chaining) queries: the oracle's restatement of
src/codegen/backward.zig against hand-traced answers.  CPU only."""
import pytest

from tensor_logic_lang_b200 import abi, lang

import backward_cases as bc


@pytest.mark.parametrize("name,src,want", bc.KNOWN, ids=[k[0] for k in bc.KNOWN])
def test_oracle_known_answers(oracle_lib, name, src, want):
    r = oracle_lib.OracleRun(lang.Program(src))
    assert r.status == 0
    assert r.queries == want


@pytest.mark.parametrize("name,src,want", bc.KNOWN, ids=[k[0] for k in bc.KNOWN])
def test_oracle_builds_agree(oracle_lib, name, src, want):
    # the -O0 build mirrors the reference's unoptimised clang build
    p = lang.Program(src)
    assert oracle_lib.OracleRun(p, libname="liboracle_O0.so").queries == oracle_lib.OracleRun(p).queries


def test_forward_and_backward_queries_interleave(oracle_lib):
    r = oracle_lib.OracleRun(lang.Program(bc.MIXED))
    lines = r.queries.splitlines()
    assert [ln.split(" ")[0] for ln in lines] == ["R[16]", "R", "E[16]", "R"]
    assert lines[1] == "R = 1" and lines[3] == "R = 0"


def test_memo_is_shared_across_queries(oracle_lib):
    # the second query of an element returns the memo the first one left
    src = bc.CHAIN.replace("Ancestor[1,3]?", "Ancestor[0,3]?")
    r = oracle_lib.OracleRun(lang.Program(src))
    assert r.queries == "Ancestor = 1\nAncestor = 0\nAncestor = 1\n"


def test_query_without_equation_is_an_error(oracle_lib):
    # the reference emits a call to an undefined @compute_Q and fails to link
    r = oracle_lib.OracleRun(lang.Program(bc.NO_EQUATION))
    assert r.status == abi.TL_ERR_UNSUPPORTED


def test_out_of_range_constant_reads_zero(oracle_lib):
    r = oracle_lib.OracleRun(lang.Program(bc.OUT_OF_RANGE))
    assert r.status == 0
    assert r.queries == "Ancestor = 1\nAncestor = 0\nAncestor = 0\nAncestor = 1\n"
