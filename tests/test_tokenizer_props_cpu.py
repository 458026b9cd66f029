"""Tokenizer round trips on arbitrary text (hypothesis): the byte tokenizer and the
GGUF SentencePiece-style tokenizer (greedy longest match, and BPE merges) with a
full set of <0xNN> byte-fallback pieces decode what they encode, and the streaming
decoder emits the same text piece by piece, never splitting a UTF-8 character."""
from hypothesis import given, settings
from hypothesis import strategies as st

from openmini_v1_b200.engine.tokenizer import ByteTokenizer, GGUFTokenizer, IncrementalDecoder

SP = "▁"
BYTES = [f"<0x{b:02X}>" for b in range(256)]
WORDS = [SP + "the", SP + "a", "th", "he", "in", SP, "e", "t", "h", SP + "t", "ing", "✓", "é"]


def _gguf(merges):
    toks = ["<unk>", "<s>", "</s>"] + BYTES + WORDS
    types = [2, 3, 3] + [6] * 256 + [1] * len(WORDS)
    return GGUFTokenizer(toks, token_types=types, merges=merges)


GREEDY = _gguf(None)
BPE = _gguf([f"{SP} t", "t h", "h e", f"{SP}t he", "i n", "in g"])
text = st.text(alphabet=st.characters(blacklist_categories=("Cs",)), max_size=60)


@settings(max_examples=200, deadline=None)
@given(s=text)
def test_round_trips(s):
    bt = ByteTokenizer()
    assert bt.decode(bt.encode(s)) == s
    for tok in (GREEDY, BPE):
        ids = tok.encode(s)
        assert ids[0] == tok.bos_id and all(0 <= i < tok.vocab_size for i in ids)
        assert tok.unk_id not in ids[1:]          # every character is covered by pieces or bytes
        assert tok.decode(ids) == s, (s, ids)
        d = IncrementalDecoder(tok)
        pieces = [d.push(i) for i in ids[1:]]
        assert "".join(pieces) == s


def test_bpe_merges_apply():
    ids = BPE.encode("the thing", add_bos=False)
    assert BPE.tokens[ids[0]] == SP + "the" and SP + "t" not in [BPE.tokens[i] for i in ids[:1]]
    assert "ing" in [BPE.tokens[i] for i in ids]
