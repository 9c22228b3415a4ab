"""The grammar mirror (rust-llm_b200/grammar.py) against answers derived by
hand from src/decoder.rs:378-557, quirks included."""
import numpy as np
import pytest

import grammar

RULES = """
# comment lines and blank lines are skipped

a ::= "xy" | [5, 7, x, 9]
b ::= a | "z"
c ::= b | undefined_rule | c
d ::= "" | [65]
"""


def test_parse_variants_and_forward_references():
    g = grammar.Grammar.from_ggnf(RULES)
    assert [r.name for r in g.rules] == ["a", "b", "c", "d"]
    a, b, c, d = g.rules
    assert a.variants == [grammar.Literal("xy"), grammar.CharClass([5, 7, 9])]  # "x" is dropped
    assert b.variants == [grammar.RuleRef(0), grammar.Literal("z")]
    # an unknown name and the rule's own name (not yet defined) both refer to rule 0
    assert c.variants == [grammar.RuleRef(1), grammar.RuleRef(0), grammar.RuleRef(0)]
    assert d.variants == [grammar.Literal(""), grammar.CharClass([65])]


def test_no_rules_is_an_error():
    with pytest.raises(ValueError):
        grammar.Grammar.from_ggnf("# nothing\n\n")


def test_allowed_tokens_follow_the_oldest_of_the_last_ten():
    g = grammar.Grammar.from_ggnf(RULES)
    x, z = ord("x"), ord("z")
    assert g.get_allowed_tokens([]) == []  # no rule active
    # token 'x' activates rule a (literal "xy" starts with 'x'): its literals and class
    assert g.get_allowed_tokens([x]) == sorted({x, ord("y"), 5, 7, 9})
    # token 0 activates every rule holding a reference to rule 0 (b and c)
    assert g.get_allowed_tokens([0]) == sorted({0, z, 1})
    # token 'z' activates b
    assert g.get_allowed_tokens([z]) == [0, z]
    # only the oldest of the last ten tokens decides
    assert g.get_allowed_tokens([1, 2, 3, x] + [99] * 9) == g.get_allowed_tokens([x])
    assert g.get_allowed_tokens([x] + [99] * 10) == []  # x is eleventh from the end
    # token 1 activates c (it refers to rule 1)
    assert g.get_allowed_tokens([1]) == [0, 1]


def test_mask_row():
    g = grammar.Grammar.from_ggnf(RULES)
    m = g.mask([ord("x")], 100)
    ids = [i for i in range(100) if (m[i >> 5] >> (i & 31)) & 1]
    assert ids == [5, 7, 9]  # 'x' (120) and 'y' (121) are past V = 100
    assert m.dtype == np.uint32 and m.shape == (4,)
