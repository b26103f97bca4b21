"""The `.tl` reader: statement forms and the reference's expression precedence."""
import pytest

from tensor_logic_lang_b200 import abi, lang


def test_implicit_product_binds_loosest():
    # `Q K / 8.0` is Q * (K / 8.0) (parser.zig:485-500)
    (eq,) = lang.parse("S[q,k] = Q[q,d] K[k,d] / 8.0\n")
    assert eq[0] == "eq" and eq[3][0] == "prod"
    assert eq[3][2][0] == "bin" and eq[3][2][1] == "/"


def test_three_factor_product_is_left_nested():
    (eq,) = lang.parse("H[v,f] = relu(A[v,u] X[u,g] W[g,f])\n")
    nl = eq[3]
    assert nl[0] == "nl" and nl[1] == "relu"
    assert nl[2][0] == "prod" and nl[2][1][0] == "prod"


def test_index_forms():
    (eq,) = lang.parse("Y[i/2, j., k'] avg= X[i+1, j-2, 3, 0:4, *t, k']\n")
    lhs = eq[1][2]
    assert [ix[0] for ix in lhs] == [abi.IX_DIV, abi.IX_NORMALIZE, abi.IX_PRIMED]
    rhs = eq[3][2]
    assert [ix[0] for ix in rhs] == [abi.IX_ADD, abi.IX_SUB, abi.IX_CONST, abi.IX_SLICE, abi.IX_VIRTUAL,
                                     abi.IX_PRIMED]
    assert eq[2] == "avg="


@pytest.mark.parametrize("op", ["=", "+=", "*=", "max=", "min=", "avg="])
def test_accumulation_ops(op):
    (eq,) = lang.parse(f"A[i] {op} B[i]\n")
    assert eq[2] == op


def test_statements():
    src = ('domain n: 5\nsparse E[n, n]\nR[x,y] = step(E[x,y])\nsave R "r.bin"\nload R "r.bin"\n'
           'backward L wrt W1, W2\nR?\n')
    kinds = [s[0] for s in lang.parse(src)]
    assert kinds == ["domain", "sparse", "eq", "save", "load", "backward", "query"]


def test_lowering_postfix():
    eq = lang.lower_equation(lang.parse("Y[b,o] = sigmoid(Z[b,o], 0.5) - T[b,o]\n")[0])
    ops = [eq.code[k].op for k in range(eq.n_code)]
    assert ops == [abi.OP_REF, abi.OP_NL, abi.OP_REF, abi.OP_SUB]
    assert eq.code[1].arg2 == 1 and eq.code[1].value == 0.5
    assert eq.refs[0].tensor == b"Z" and eq.refs[1].tensor == b"T"


def test_paren_then_identifier_is_not_a_group():
    # parser.zig:688-697: `(` followed by an identifier is a relation, not a group
    with pytest.raises(lang.ParseError):
        lang.parse("L[n] = (Y[n] - T[n]) * (Y[n] - T[n])\n")
