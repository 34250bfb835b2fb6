"""Byte tokenizer and greedy generation shapes."""

from underhfs.nn import TransformerLM
from underhfs.text import ByteTokenizer


def test_byte_roundtrip():
    tok = ByteTokenizer()
    assert tok.decode(tok.encode("underHFS on B200")) == "underHFS on B200"


def test_generate_appends_valid_tokens():
    lm = TransformerLM(vocab_size=256, max_seq_len=8, features=4, hidden_features=8, layers=1)
    out = lm.generate(ByteTokenizer().encode("hi"), max_new_tokens=3)
    assert out.shape == (5,)
    assert all(0 <= v < 256 for v in out._storage)


def test_generate_truncates_context_to_max_seq_len():
    lm = TransformerLM(vocab_size=256, max_seq_len=4, features=4, hidden_features=8, layers=1)
    out = lm.generate(ByteTokenizer().encode("abcdef"), max_new_tokens=2)
    assert out.shape == (8,)
