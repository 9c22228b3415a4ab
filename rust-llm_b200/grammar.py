"""The reference's grammar (src/decoder.rs:378-557), same names and results,
emitting the bit-packed allowed mask the device sampler takes. (The two
builders create_json_grammar / create_code_grammar, :559-602, stay in the
Rust crate: they only feed their rule text to Grammar::from_ggnf.)

Grammar.from_ggnf parses one rule per line (`name ::= v1 | v2 ...`); a
variant is a literal (`"..."`), a class of numeric ids (`[1,2,3]`; anything
that does not parse as an id is dropped), or a reference to a rule defined
on an EARLIER line (anything else refers to rule 0). get_allowed_tokens
replays the last ten tokens newest first, each replay replacing the state,
so the state is that of the oldest of them: the rules with a literal whose
first character code, or a rule reference whose index, equals that token.
The allowed ids are the active rules' literal character codes, class ids and
referenced indices, sorted and deduplicated. These are the reference's
semantics, quirks included (src/decoder.rs:466-528); Sampler.with_grammar
(decoder.py) turns them into a mask row for rl_grammar_greedy_host, and an
empty set allows every id as in Sampler::sample_with_grammar.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


@dataclass
class Literal:
    text: str


@dataclass
class RuleRef:
    index: int


@dataclass
class CharClass:
    ids: list


@dataclass
class GrammarRule:
    name: str
    variants: list = field(default_factory=list)


def _parse_id(x: str):
    """Rust's `x.trim().parse::<usize>().ok()`: decimal digits, an optional
    leading '+', no sign, no whitespace inside."""
    t = x.strip()
    if t.startswith("+"):
        t = t[1:]
    return int(t) if t.isdigit() and t.isascii() else None


class Grammar:
    def __init__(self):
        self.rules: list[GrammarRule] = []
        self.start_rule = 0
        self.name_to_idx: dict[str, int] = {}

    @classmethod
    def from_ggnf(cls, ggnf: str) -> "Grammar":
        """Grammar::from_ggnf (src/decoder.rs:393-397); ValueError where the
        reference returns Err."""
        g = cls()
        g._parse_ggnf(ggnf)
        return g

    def _parse_ggnf(self, ggnf: str):
        for line in ggnf.splitlines():
            line = line.strip()
            if not line or line.startswith("#"):
                continue
            if "::=" not in line:
                continue
            name, definition = line.split("::=", 1)
            name = name.strip()
            variants = [self._parse_variant(part) for part in definition.strip().split("|")]
            idx = len(self.rules)
            self.name_to_idx[name] = idx  # after the variants: a rule cannot name itself
            self.rules.append(GrammarRule(name, variants))
        if not self.rules:
            raise ValueError("No rules found in grammar")

    def _parse_variant(self, s: str):
        s = s.strip()
        if s.startswith('"') and s.endswith('"'):
            if len(s) < 2:
                raise ValueError(f"a one-character literal {s!r} (the reference's slice panics here)")
            return Literal(s[1:-1])
        if s.startswith("[") and s.endswith("]"):
            ids = [_parse_id(x) for x in s[1:-1].split(",")]
            return CharClass([i for i in ids if i is not None])
        return RuleRef(self.name_to_idx.get(s, 0))

    @staticmethod
    def _matches(variant, token: int) -> bool:
        if isinstance(variant, Literal):
            return bool(variant.text) and ord(variant.text[0]) == token
        if isinstance(variant, RuleRef):
            return variant.index == token
        return False

    def get_allowed_tokens(self, prev_tokens) -> list:
        """Grammar::get_allowed_tokens (src/decoder.rs:466-473)."""
        state = [False] * len(self.rules)
        for token in list(prev_tokens)[::-1][:10]:
            state = [any(self._matches(v, int(token)) for v in r.variants) for r in self.rules]
        allowed = set()
        for idx, active in enumerate(state):
            if not active:
                continue
            for v in self.rules[idx].variants:
                if isinstance(v, Literal):
                    allowed.update(ord(c) for c in v.text)
                elif isinstance(v, CharClass):
                    allowed.update(v.ids)
                elif isinstance(v, RuleRef):
                    allowed.add(v.index)
        return sorted(allowed)

    def mask(self, prev_tokens, V: int) -> np.ndarray:
        """The allowed ids as one bit-packed mask row for a vocabulary of V
        (bit j of word w is id 32w + j; ids >= V dropped)."""
        from decoder import allowed_mask

        return allowed_mask(self.get_allowed_tokens(prev_tokens), V)


# ---------------------------------------------------------------------------
# Real GBNF grammars (the step after the toy automaton above): compiled in the
# native library (rl_gbnf_*), masks written as the bit-packed rows the device
# samplers take.
# ---------------------------------------------------------------------------
class GbnfState:
    """One sequence's position in a Gbnf grammar (rl_gbnf_state)."""

    def __init__(self, grammar: "Gbnf", handle):
        self.grammar = grammar
        self.h = handle

    def copy(self) -> "GbnfState":
        import rlsampler

        s = self.grammar.new_state()
        rlsampler.check(rlsampler.lib().rl_gbnf_state_copy(self.h, s.h), "rl_gbnf_state_copy")
        return s

    @property
    def accepting(self) -> bool:
        import rlsampler

        return bool(rlsampler.lib().rl_gbnf_accepting(self.h))

    def __del__(self):
        try:
            import rlsampler

            if self.h:
                rlsampler.lib().rl_gbnf_state_destroy(self.h)
                self.h = None
        except Exception:
            pass


class Gbnf:
    """A GBNF grammar compiled against a vocabulary (token texts as bytes).

    mask(state) -> (row, n): the allowed tokens as one bit-packed uint32 row
    (bit j of word w is token 32w + j) and their count; accept(state, token)
    advances the state (RLError when the grammar does not allow the token).
    The end-of-sequence id is allowed exactly when the start rule is complete."""

    def __init__(self, text: str, tokens, eos_id: int = -1, root: str = "root"):
        import ctypes

        import rlsampler

        toks = [t.encode() if isinstance(t, str) else bytes(t) for t in tokens]
        self.V = len(toks)
        self.words = (self.V + 31) // 32
        self.eos_id = eos_id
        bufs = [ctypes.create_string_buffer(t, max(len(t), 1)) for t in toks]
        ptrs = (ctypes.c_void_p * self.V)(*[ctypes.cast(b, ctypes.c_void_p) for b in bufs])
        lens = np.array([len(t) for t in toks], np.int32)
        h = ctypes.c_void_p()
        rlsampler.check(rlsampler.lib().rl_gbnf_create(text.encode(), root.encode(), self.V, ptrs,
                                                       lens.ctypes.data_as(ctypes.c_void_p), eos_id,
                                                       ctypes.byref(h)), "rl_gbnf_create")
        self.h = h

    def new_state(self) -> GbnfState:
        import ctypes

        import rlsampler

        h = ctypes.c_void_p()
        rlsampler.check(rlsampler.lib().rl_gbnf_state_create(self.h, ctypes.byref(h)), "rl_gbnf_state_create")
        return GbnfState(self, h)

    def mask(self, state: GbnfState):
        import ctypes

        import rlsampler

        row = np.zeros(self.words, np.uint32)
        n = ctypes.c_int32()
        rlsampler.check(rlsampler.lib().rl_gbnf_mask(self.h, state.h, row.ctypes.data_as(ctypes.c_void_p),
                                                     self.words, ctypes.byref(n)), "rl_gbnf_mask")
        return row, n.value

    def mask_batch(self, states, out=None, nthreads: int = 8):
        """Rows for every state into out [len(states), words] (uint32)."""
        import ctypes

        import rlsampler

        B = len(states)
        if out is None:
            out = np.zeros((B, self.words), np.uint32)
        n = np.zeros(B, np.int32)
        hs = (ctypes.c_void_p * max(B, 1))(*[s.h for s in states])
        rlsampler.check(rlsampler.lib().rl_gbnf_mask_batch(self.h, hs, B, out.ctypes.data_as(ctypes.c_void_p),
                                                           out.shape[1], n.ctypes.data_as(ctypes.c_void_p),
                                                           nthreads), "rl_gbnf_mask_batch")
        return out, n

    def accept(self, state: GbnfState, token: int):
        import rlsampler

        rlsampler.check(rlsampler.lib().rl_gbnf_accept(self.h, state.h, int(token)), "rl_gbnf_accept")

    def accept_batch(self, states, tokens, nthreads: int = 8):
        """accept() for every state and its token (rows over host threads);
        RLError if any row's token is refused (those rows stay unchanged)."""
        import ctypes

        import rlsampler

        B = len(states)
        toks = np.ascontiguousarray(tokens, np.int32)
        st = np.zeros(B, np.int32)
        hs = (ctypes.c_void_p * max(B, 1))(*[s.h for s in states])
        rlsampler.check(rlsampler.lib().rl_gbnf_accept_batch(self.h, hs, toks.ctypes.data_as(ctypes.c_void_p), B,
                                                             st.ctypes.data_as(ctypes.c_void_p), nthreads),
                        "rl_gbnf_accept_batch")
        return st

    def allowed(self, state: GbnfState):
        """The allowed token ids (sorted)."""
        row, _ = self.mask(state)
        bits = np.unpackbits(row.view(np.uint8), bitorder="little")[: self.V]
        return np.flatnonzero(bits).tolist()

    def __del__(self):
        try:
            import rlsampler

            if self.h:
                rlsampler.lib().rl_gbnf_destroy(self.h)
                self.h = None
        except Exception:
            pass
