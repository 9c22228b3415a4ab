"""Real GBNF token masks (rl_gbnf_*, grammar.Gbnf): the compiled automaton
against an independent oracle, on the host (no GPU).

- Non-recursive grammars: each is paired with a hand-written regular
  expression of the same language; a token t is allowed after the text P
  exactly when regex.fullmatch(pattern, P + t, partial=True) succeeds (some
  continuation of P + t is in the language), and the end-of-sequence id
  exactly when P itself is in it. Random walks over random vocabularies
  compare the whole mask at every step.
- A recursive grammar (JSON): random documents, split greedily into tokens
  of the vocabulary, are accepted token by token, each token in the mask
  before it is accepted, with the end token allowed exactly at the end;
  damaged documents are refused at the damage.
- Errors: syntax, undefined rules, left recursion, disallowed tokens.
"""
import json

import numpy as np
import pytest
import regex

import grammar
import rlsampler
import workloads

ALPHABET = "abcxyz0123456789.,[]{}\":- truefalsnhiloABZ\\"


def vocab(rng, n, words=()):
    toks = set(ALPHABET) | set(words)
    while len(toks) < n:
        k = int(rng.integers(2, 5))
        toks.add("".join(rng.choice(list(ALPHABET), k)))
    toks = sorted(toks)
    return toks + [""]  # the last id is the end token (no bytes)


CASES = [
    # (grammar, equivalent regex)
    ('root ::= ("true" | "false" | [0-9]+ ("." [0-9]+)?)', r"(?:true|false|[0-9]+(?:\.[0-9]+)?)"),
    ('root ::= "[" ( item ( "," item )* )? "]"\nitem ::= [a-c]{1,3}', r"\[(?:[a-c]{1,3}(?:,[a-c]{1,3})*)?\]"),
    ('root ::= greeting " " name   # a comment\ngreeting ::= "hi"\n         | "hello"\nname ::= [A-Z] [a-z]*',
     r"(?:hi|hello) [A-Z][a-z]*"),
    ('root ::= "\\"" [^"\\\\]* "\\""', r'"[^"\\]*"'),
    ('root ::= x{2} y? x{0,2}\nx ::= "ab" | "c"\ny ::= [0-9]{1,}', r"(?:ab|c){2}(?:[0-9]{1,})?(?:ab|c){0,2}"),
    ('root ::= ( "a" | "b" )+ "." ( [xyz] "," )*', r"(?:a|b)+\.(?:[xyz],)*"),
]


def oracle_mask(pattern, prefix, toks, eos):
    allowed = set()
    for t, s in enumerate(toks):
        if t == eos or not s:
            continue
        if regex.fullmatch(pattern, prefix + s, partial=True) is not None:
            allowed.add(t)
    if regex.fullmatch(pattern, prefix) is not None:
        allowed.add(eos)
    return allowed


@pytest.mark.parametrize("case", range(len(CASES)))
def test_masks_equal_the_regex_oracle(case):
    text, pattern = CASES[case]
    rng = np.random.default_rng(100 + case)
    toks = vocab(rng, 300, words=("true", "false", "hello", "hi", "ab", "12", "3.5"))
    eos = len(toks) - 1
    g = grammar.Gbnf(text, toks, eos_id=eos)
    for walk in range(6):
        s = g.new_state()
        prefix = ""
        for step in range(25):
            got = set(g.allowed(s))
            want = oracle_mask(pattern, prefix, toks, eos)
            assert got == want, (case, walk, step, repr(prefix), sorted(got ^ want)[:10])
            assert s.accepting == (eos in want)
            choices = sorted(want - {eos})
            if not choices:
                break
            t = int(rng.choice(choices))
            g.accept(s, t)
            prefix += toks[t]


JSON = workloads.GBNF_JSON


def random_json(rng, depth=0):
    k = int(rng.integers(0, 7 if depth < 3 else 4))
    if k == 0:
        return int(rng.integers(-1000, 1000))
    if k == 1:
        return float(np.round(rng.normal(0, 100), 3))
    if k == 2:
        return "".join(rng.choice(list("abc xyz\"\\/\né"), int(rng.integers(0, 8))))
    if k == 3:
        return [True, False, None][int(rng.integers(0, 3))]
    if k in (4, 5):
        return [random_json(rng, depth + 1) for _ in range(int(rng.integers(0, 4)))]
    return {"".join(rng.choice(list("abkey"), 3)): random_json(rng, depth + 1) for _ in range(int(rng.integers(0, 4)))}


def greedy_tokens(text, toks_by_len):
    """Longest-match split of the text's bytes into vocabulary tokens."""
    b = text.encode()
    out, i = [], 0
    while i < len(b):
        for L in range(min(8, len(b) - i), 0, -1):
            t = toks_by_len.get(b[i:i + L])
            if t is not None:
                out.append(t)
                i += L
                break
        else:
            raise AssertionError("no token for byte %r" % b[i:i + 1])
    return out


def json_vocab(rng):
    words = ['{"', '":', '",', '"}', "true", "false", "null", "[", "]", "{}", "[]", ", ", ": ", "\\n", "\\u00",
             "12", "0.", "e+", "-1"]
    toks = [bytes([c]) for c in range(256)] + [w.encode() for w in words]
    while len(toks) < 600:
        toks.append("".join(rng.choice(list("abkey\":,{}[]0123456789. "), int(rng.integers(2, 5)))).encode())
    toks = list(dict.fromkeys(toks))
    return toks + [b""]


def test_json_documents_are_accepted_token_by_token():
    rng = np.random.default_rng(7)
    toks = json_vocab(rng)
    eos = len(toks) - 1
    by = {t: i for i, t in enumerate(toks) if t}
    g = grammar.Gbnf(JSON, toks, eos_id=eos)
    for n in range(40):
        doc = json.dumps(random_json(rng), separators=(",", ":") if n % 2 else (", ", ": "))
        s = g.new_state()
        for t in greedy_tokens(doc, by):
            assert t in set(g.allowed(s)), (doc, toks[t])
            g.accept(s, t)
        assert s.accepting and eos in set(g.allowed(s)), doc
        g.accept(s, eos)
        row, cnt = g.mask(s)
        assert cnt == 0 and not row.any()


def test_damaged_json_is_refused():
    rng = np.random.default_rng(8)
    toks = json_vocab(rng)
    eos = len(toks) - 1
    by = {t: i for i, t in enumerate(toks) if t}
    g = grammar.Gbnf(JSON, toks, eos_id=eos)
    s = g.new_state()
    for t in greedy_tokens('{"a": [1, 2', by):
        g.accept(s, t)
    assert not s.accepting and eos not in set(g.allowed(s))  # unfinished
    assert by[b"}"] not in set(g.allowed(s))  # the array is still open
    with pytest.raises(rlsampler.RLError) as e:
        g.accept(s, by[b"}"])
    assert e.value.status == rlsampler.RL_ERR_INVALID_ARG
    g.accept(s, by[b"]"])  # the state was left unchanged by the refusal
    g.accept(s, by[b"}"])
    assert s.accepting


def test_batch_masks_and_state_copies():
    rng = np.random.default_rng(9)
    toks = json_vocab(rng)
    eos = len(toks) - 1
    by = {t: i for i, t in enumerate(toks) if t}
    g = grammar.Gbnf(JSON, toks, eos_id=eos)
    states = []
    for n in range(12):
        s = g.new_state()
        doc = json.dumps(random_json(rng))
        ts = greedy_tokens(doc, by)
        for t in ts[: int(rng.integers(0, len(ts) + 1))]:
            g.accept(s, t)
        states.append(s)
    rows, counts = g.mask_batch(states, nthreads=4)
    for s, r, c in zip(states, rows, counts):
        one, n1 = g.mask(s)
        assert np.array_equal(r, one) and c == n1
    c = states[3].copy()
    before = g.allowed(states[3])
    t = g.allowed(c)[0]
    if t != eos:
        g.accept(c, t)
    assert g.allowed(states[3]) == before


@pytest.mark.parametrize("text,status", [
    ('root ::= "abc', rlsampler.RL_ERR_INVALID_ARG),          # unterminated literal
    ("root ::= missing", rlsampler.RL_ERR_INVALID_ARG),        # undefined rule
    ('root ::= "a"\nroot ::= "b"', rlsampler.RL_ERR_INVALID_ARG),  # defined twice
    ('root ::= [a-', rlsampler.RL_ERR_INVALID_ARG),           # unterminated class
    ('root ::= "\\q"', rlsampler.RL_ERR_INVALID_ARG),          # unknown escape
    ("root ::= root \"a\" | \"b\"", rlsampler.RL_ERR_UNSUPPORTED),  # left recursion
    ('root ::= x "a"\nx ::= "" | root', rlsampler.RL_ERR_UNSUPPORTED),  # through a nullable prefix
])
def test_grammar_errors(text, status):
    with pytest.raises(rlsampler.RLError) as e:
        grammar.Gbnf(text, ["a", "b", ""], eos_id=2)
    assert e.value.status == status


def test_right_recursion_does_not_deepen_the_stacks():
    g = grammar.Gbnf('root ::= "a" root | "b"', ["a", "b", ""], eos_id=2)
    s = g.new_state()
    for _ in range(5000):  # far beyond the 1024-frame stack limit
        g.accept(s, 0)
    assert g.allowed(s) == [0, 1]
    g.accept(s, 1)
    assert g.allowed(s) == [2]


UCASES = [
    # classes and '.' are over characters (code points), matched as their UTF-8 bytes
    ('root ::= [α-ω]+ "." [^a-z]', r"[α-ω]+\.[^a-z]"),
    ('root ::= "x" . "y"', r"(?s)x.y"),
    ('root ::= "\\u00e9" [\\u4e00-\\u9fff]{1,2} "\\U0001F600"?', "é[一-鿿]{1,2}(?:\U0001F600)?"),
    ('root ::= [^é中]+ "!"', r"[^é中]+!"),
]
UALPHA = list("abxy.!") + list("αβγωé中文字") + ["\U0001F600", "ÿ", "ࠀ", "\n"]


@pytest.mark.parametrize("case", range(len(UCASES)))
def test_unicode_masks_equal_the_regex_oracle(case):
    text, pattern = UCASES[case]
    rng = np.random.default_rng(200 + case)
    toks = set(UALPHA)
    while len(toks) < 200:
        toks.add("".join(rng.choice(UALPHA, int(rng.integers(2, 4)))))
    toks = sorted(toks) + [""]
    eos = len(toks) - 1
    g = grammar.Gbnf(text, toks, eos_id=eos)
    for walk in range(6):
        s = g.new_state()
        prefix = ""
        for step in range(15):
            got = set(g.allowed(s))
            want = oracle_mask(pattern, prefix, toks, eos)
            assert got == want, (case, walk, step, repr(prefix), sorted(got ^ want)[:10])
            choices = sorted(want - {eos})
            if not choices:
                break
            t = int(rng.choice(choices))
            g.accept(s, t)
            prefix += toks[t]


def test_tokens_that_split_a_character():
    """Byte-level tokens may end inside a UTF-8 sequence: the automaton
    follows the character across them."""
    toks = [b"\xc3", b"\xa9", b"x", "é".encode(), b""]
    g = grammar.Gbnf('root ::= "é" "x"', toks, eos_id=4)
    s = g.new_state()
    assert g.allowed(s) == [0, 3]
    g.accept(s, 0)
    assert g.allowed(s) == [1]
    g.accept(s, 1)
    assert g.allowed(s) == [2]
    g.accept(s, 2)
    assert g.allowed(s) == [4]


def test_accept_batch_equals_single_accepts():
    rng = np.random.default_rng(10)
    toks = json_vocab(rng)
    eos = len(toks) - 1
    by = {t: i for i, t in enumerate(toks) if t}
    g = grammar.Gbnf(JSON, toks, eos_id=eos)
    docs = [greedy_tokens(json.dumps(random_json(rng)), by) for _ in range(40)]
    a = [g.new_state() for _ in docs]
    b = [g.new_state() for _ in docs]
    for step in range(max(len(d) for d in docs)):
        live = [i for i, d in enumerate(docs) if step < len(d)]
        g.accept_batch([a[i] for i in live], [docs[i][step] for i in live], nthreads=4)
        for i in live:
            g.accept(b[i], docs[i][step])
    for x, y in zip(a, b):
        assert g.allowed(x) == g.allowed(y) and x.accepting
    # a refused token: that row's status, the others advance
    s1, s2 = g.new_state(), g.new_state()
    with pytest.raises(rlsampler.RLError):
        g.accept_batch([s1, s2], [by[b"{"], by[b"}"]])
    assert g.allowed(s2) == g.allowed(g.new_state())
    assert by[b"}"] in set(g.allowed(s1))  # s1 took '{'


def test_accept_automaton_past_its_bound():
    """More distinct states than the accept path's lazy automaton keeps
    (16,384): it is emptied and refilled on the way, and the states walk on
    exactly as a second grammar's do."""
    toks = [chr(c) for c in range(ord("a"), ord("z") + 1)] + [""]
    eos = len(toks) - 1
    text = 'root ::= ("a" [b-z]{0,60}){0,1000}'  # unambiguous: 'a' always opens a group
    g1 = grammar.Gbnf(text, toks, eos_id=eos)
    g2 = grammar.Gbnf(text, toks, eos_id=eos)
    rng = np.random.default_rng(12)
    s1, s2 = g1.new_state(), g2.new_state()
    for step in range(20000):
        allowed = [t for t in g1.allowed(s1) if t != eos]
        if not allowed:
            break
        rest = [x for x in allowed if x != 0]
        t = 0 if (not rest or rng.random() < 0.03) else int(rng.choice(rest))  # a new group now and then
        g1.accept(s1, t)
        g2.accept(s2, t)
        if step % 997 == 0:
            assert g1.allowed(s1) == g2.allowed(s2)
    assert step > 16384
    assert g1.allowed(s1) == g2.allowed(s2) and s1.accepting == s2.accepting


def test_generated_documents_parse_as_json():
    """Random walks through the masks (any allowed token; after a while the
    closing tokens and the end token are preferred) end only in documents
    that json.loads accepts."""
    rng = np.random.default_rng(13)
    toks = json_vocab(rng)
    eos = len(toks) - 1
    g = grammar.Gbnf(JSON, toks, eos_id=eos)
    closers = {i for i, t in enumerate(toks) if t in (b"]", b"}", b'"', b"0", b"1")}
    finished = 0
    for walk in range(60):
        s = g.new_state()
        text = b""
        for step in range(400):
            allowed = g.allowed(s)
            if step > 20:
                pref = [t for t in allowed if t == eos or t in closers]
                if pref:
                    allowed = pref
            t = eos if eos in allowed and step > 20 else int(rng.choice(allowed))
            g.accept(s, t)
            if t == eos:
                json.loads(text.decode("utf-8", errors="surrogateescape"))
                finished += 1
                break
            text += toks[t]
    assert finished >= 50
