"""The text front end (tensai_b200/tokenizer.py) against the reference
tokenizer's own known answers (tokenizer/tokenizer_test.go: its tiny
byte-level BPE fixture) and against the Hugging Face `tokenizers` library,
which the reference verifies itself against (tokenizer/verify_hf.py), on
tokenizers trained here with both pre-tokenization patterns. CPU only."""
import json

import pytest

from tensai_b200.tokenizer import Parse

GPT2_PRE = {"type": "ByteLevel", "add_prefix_space": False, "trim_offsets": True}
CL100K_RE = ("(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\\r\\n\\p{L}\\p{N}]?\\p{L}+|\\p{N}| ?[^\\s\\p{L}\\p{N}]+[\\r\\n]*|"
             "\\s*[\\r\\n]+|\\s+(?!\\S)|\\s+")
CL100K3_RE = CL100K_RE.replace("\\p{N}|", "\\p{N}{1,3}|", 1)  # digits in runs of up to 3
CL100K_PRE = {"type": "Sequence", "pretokenizers": [
    {"type": "Split", "pattern": {"Regex": CL100K_RE}, "behavior": "Isolated", "invert": False},
    {"type": "ByteLevel", "add_prefix_space": False, "trim_offsets": False, "use_regex": False}]}
STRING_MERGES = ["h e", "l l", "he ll", "hell o", "1 2", "12 3"]
PAIR_MERGES = [["h", "e"], ["l", "l"], ["he", "ll"], ["hell", "o"], ["1", "2"], ["12", "3"]]


def fixture(pre, merges):
    """The reference test's tokenizer.json (Ġ, U+0120, stands for a space)."""
    return json.dumps({
        "added_tokens": [{"id": 12, "content": "<|end|>", "special": True}],
        "normalizer": None,
        "pre_tokenizer": pre,
        "model": {"type": "BPE",
                  "vocab": {"h": 0, "e": 1, "l": 2, "o": 3, "Ġ": 4, "1": 5, "2": 6, "3": 7, "he": 8, "ll": 9,
                            "hell": 10, "hello": 11, "12": 13, "123": 14},
                  "merges": merges}})


@pytest.mark.parametrize("merges", [STRING_MERGES, PAIR_MERGES])
def test_encode_decode(merges):
    tok = Parse(fixture(GPT2_PRE, merges))
    got = tok.Encode("hello hello")
    assert got == [11, 4, 11]  # " hello" keeps its leading space, whose Ġ does not merge
    assert tok.Decode(got) == "hello hello"


def test_special_tokens():
    tok = Parse(fixture(GPT2_PRE, STRING_MERGES))
    got = tok.Encode("hello<|end|>hello")
    assert got == [11, 12, 11]
    assert tok.Decode(got) == "hello<|end|>hello"
    assert tok.ID("<|end|>") == (12, True)
    assert tok.Len() == 15


def test_digit_splitting():
    assert Parse(fixture(GPT2_PRE, STRING_MERGES)).Encode("123") == [14]  # one pre-token: merges build "123"
    assert Parse(fixture(CL100K_PRE, STRING_MERGES)).Encode("123") == [5, 6, 7]  # \p{N} isolates each digit


def test_parse_errors():
    with pytest.raises(ValueError):
        Parse("{")
    with pytest.raises(ValueError, match="unsupported pre_tokenizer"):
        Parse(fixture({"type": "Whitespace"}, STRING_MERGES))
    with pytest.raises(ValueError, match="unsupported split pattern"):
        Parse(fixture({"type": "Split", "pattern": {"Regex": "[a-z]+"}}, STRING_MERGES))
    bad = {"normalizer": {"type": "Lowercase"}, "pre_tokenizer": GPT2_PRE,
           "model": {"type": "BPE", "vocab": {"a": 0}, "merges": []}}
    with pytest.raises(ValueError, match="unsupported normalizer"):
        Parse(json.dumps(bad))
    nfc = dict(bad, normalizer={"type": "NFC"})
    Parse(json.dumps(nfc))  # NFC passes through


# ---- against Hugging Face tokenizers -------------------------------------------

CORPUS = [
    "The quick brown fox jumps over the lazy dog. It's 2024; they'll say it's fine.",
    "Numbers 12345 and 6789, prices like $3.50 or 1,000,000 units!",
    "Tabs\tand   multiple spaces,\nnew lines\r\nand trailing spaces   ",
    "Café naïve résumé über straße Ångström",
    "Привет мир, こんにちは世界, "
    "مرحبا",
    "Emoji \U0001F600\U0001F680 and symbols ∑∞≠ ½ Ⅳ ٣٤",
    "I'M SHOUTING, YOU'RE NOT. We'Ve seen 'quotes' and \"double quotes\".",
    "code: def f(x): return x**2 + 3*x - 1  # comment\n\n\n    indented()",
    "a b c　d e",
]
TESTS = CORPUS + [
    "unseen words: zyxwvut qqq 987654321000 ...!!! ???",
    "  leading spaces and\n\n\nblank lines\n",
    "mixed<|end|>special<|end|><|end|>tokens",
    "x'sy 'll 'D 'Re",
    "",
    " ",
    "\n",
    "é café ño",  # combining marks (category M)
    "\U0001F468‍\U0001F469‍\U0001F467 family",  # a zero-width-joiner sequence
    "no break space and em space",
    "\r\n\r\nwindows\r\nlines\r\n",
    "\t\tindent\n\t  mixed \n",
    "12345678901234567890 and ١٢٣٤٥ and ⅫⅬ",
    "'quotes'' it''s rock'n'roll ''",
    "中文字符和English混合123",
    "!!!\n\n???   ...\r\n",
    "trailing space ",
    "   ",
]


def _train(pre_tokenizer):
    tk = pytest.importorskip("tokenizers")
    from tokenizers import Tokenizer, models, pre_tokenizers, trainers
    tok = Tokenizer(models.BPE())
    if pre_tokenizer == "gpt2":
        tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    else:
        rx = CL100K_RE if pre_tokenizer == "cl100k" else CL100K3_RE
        tok.pre_tokenizer = pre_tokenizers.Sequence([
            pre_tokenizers.Split(tk.Regex(rx), behavior="isolated"),
            pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    trainer = trainers.BpeTrainer(vocab_size=600, initial_alphabet=pre_tokenizers.ByteLevel.alphabet(),
                                  special_tokens=["<|end|>"], show_progress=False)
    tok.train_from_iterator(CORPUS * 20, trainer=trainer)
    return tok


@pytest.mark.parametrize("pre", ["gpt2", "cl100k", "cl100k_digits3"])
def test_matches_hf_tokenizers(pre):
    hf = _train(pre)
    ours = Parse(hf.to_str())
    for s in TESTS:
        want = hf.encode(s).ids
        got = ours.Encode(s)
        assert got == want, (pre, s, got, want)
        assert ours.Decode(got) == s, (pre, s)
    # Go's Len: vocabulary entries plus added tokens (a special token that is
    # also in the vocabulary, as the trainer puts it, counts twice)
    f = json.loads(hf.to_str())
    assert ours.Len() == len(f["model"]["vocab"]) + len(f["added_tokens"])
