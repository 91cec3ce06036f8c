"""Byte-level BPE tokenizer for the decode engines' text front end: the Go
API of tensai's tokenizer package (tokenizer/tokenizer.go:78-297) in Python,
host-side string processing (nothing here touches the GPU).

Loads a Hugging Face tokenizer.json of the byte-level BPE family (GPT-2,
Llama 3, Qwen): the vocabulary, the merges (as "a b" strings or ["a", "b"]
pairs), the added (special) tokens and one of the two pre-tokenization
patterns found in such files, which are implemented as scanners because they
need lookahead and inline case-insensitive groups:
  * the GPT-2 split ('s|'t|'re|'ve|'m|'ll|'d| ?\\p{L}+| ?\\p{N}+|
    ?[^\\s\\p{L}\\p{N}]+|\\s+(?!\\S)|\\s+), ByteLevel's built-in regex;
  * the cl100k-style split (case-insensitive contractions, an optional
    non-letter prefix before letters, digits in runs of at most 1 or 3,
    newline runs after punctuation and "\\s*[\\r\\n]+").
Any other pattern, a normalizer other than NFC (passed through) or a model
other than BPE is rejected, as the Go package does (tokenizer.go:86-205).
Letters, numbers and white space follow Go's unicode.IsLetter (category L),
unicode.IsNumber (category N) and unicode.IsSpace (the Unicode White_Space
property). Decode returns text; byte sequences that are not UTF-8 become
U+FFFD (the Go string keeps the raw bytes).
"""
from __future__ import annotations

import json
import unicodedata

__all__ = ["Tokenizer", "Load", "Parse"]

# Unicode White_Space (PropList.txt): what Go's unicode.IsSpace accepts.
_WHITE_SPACE = frozenset([0x09, 0x0A, 0x0B, 0x0C, 0x0D, 0x20, 0x85, 0xA0, 0x1680, *range(0x2000, 0x200B), 0x2028,
                          0x2029, 0x202F, 0x205F, 0x3000])
_CONTRACTIONS = ("'s", "'t", "'re", "'ve", "'m", "'ll", "'d")


def _is_letter(c: str) -> bool:
    return unicodedata.category(c)[0] == "L"


def _is_number(c: str) -> bool:
    return unicodedata.category(c)[0] == "N"


def _is_space(c: str) -> bool:
    return ord(c) in _WHITE_SPACE


def _is_punct(c: str) -> bool:
    return not _is_space(c) and not _is_letter(c) and not _is_number(c)


class _Split:
    """Which scanner (tokenizer.go:40-51): GPT-2's or the cl100k-style one."""

    def __init__(self, ci_contractions=False, letter_prefix=False, max_digits=0, newline_runs=False):
        self.ci_contractions = ci_contractions
        self.letter_prefix = letter_prefix
        self.max_digits = max_digits
        self.newline_runs = newline_runs


def _gpt2() -> _Split:
    return _Split()


def _cl100k(max_digits: int) -> _Split:
    return _Split(True, True, max_digits, True)


def _classify_regex(re: str) -> _Split:
    if re.startswith("'s|'t|'re|'ve|'m|'ll|'d"):
        return _gpt2()
    if re.startswith("(?i:'s|'t|'re|'ve|'m|'ll|'d)"):
        return _cl100k(3 if "\\p{N}{1,3}" in re else 1)
    raise ValueError(f"tokenizer: unsupported split pattern {re!r}")


def _detect_split(pre) -> _Split:
    if pre is None:
        raise ValueError("tokenizer: missing pre_tokenizer")
    kind = pre.get("type")
    if kind == "ByteLevel":
        if pre.get("use_regex", True) is not False:
            return _gpt2()  # ByteLevel's built-in regex is the GPT-2 split
        raise ValueError("tokenizer: ByteLevel without a split pattern")
    if kind == "Sequence":
        for sub in pre.get("pretokenizers") or []:
            if isinstance(sub, dict) and sub.get("type") == "Split":
                rx = (sub.get("pattern") or {}).get("Regex", "")
                if rx:
                    return _classify_regex(rx)
        raise ValueError("tokenizer: no Split pattern in pre_tokenizer sequence")
    if kind == "Split":
        return _classify_regex((pre.get("pattern") or {}).get("Regex", ""))
    raise ValueError(f"tokenizer: unsupported pre_tokenizer type {kind!r}")


def _byte_encoder():
    """bytes_to_unicode: printable bytes stand for themselves, the others map
    to 256 and up in byte order (tokenizer.go:137-148)."""
    enc, n = [], 0
    for b in range(256):
        if ord("!") <= b <= ord("~") or 0xA1 <= b <= 0xAC or 0xAE <= b <= 0xFF:
            enc.append(chr(b))
        else:
            enc.append(chr(256 + n))
            n += 1
    return enc


class Tokenizer:
    """Encodes text to token ids and back (tokenizer.go:27-38)."""

    def __init__(self, vocab: dict, ranks: dict, specials: list, split: _Split):
        self._vocab = vocab
        self._inverse = {i: s for s, i in vocab.items()}
        self._ranks = ranks
        # longest first, so overlapping specials resolve to the longest
        self._specials = sorted(specials, key=lambda sp: -len(sp[0]))
        self._by_id = {i: s for s, i in specials}
        self._split_cfg = split
        self._byte_enc = _byte_encoder()
        self._byte_dec = {c: b for b, c in enumerate(self._byte_enc)}
        self._cache: dict[str, list[int]] = {}

    def Len(self) -> int:
        """Ids the tokenizer can produce, added tokens included."""
        return len(self._vocab) + len(self._by_id)

    def ID(self, content: str):
        """(id, True) for a token's content (special tokens first), else (0, False)."""
        for s, i in self._specials:
            if s == content:
                return i, True
        if content in self._vocab:
            return self._vocab[content], True
        return 0, False

    def Encode(self, s: str) -> list[int]:
        """Token ids of s; special tokens in the text are matched as themselves."""
        ids: list[int] = []
        while s:
            cut, cut_end, cut_id = len(s), len(s), -1
            for content, i in self._specials:
                k = s.find(content)
                if 0 <= k < cut:
                    cut, cut_end, cut_id = k, k + len(content), i
            ids.extend(self._encode_text(s[:cut]))
            if cut_id >= 0:
                ids.append(cut_id)
            s = s[cut_end:]
        return ids

    def Decode(self, ids) -> str:
        """Text of the ids (unknown ids add nothing)."""
        out = bytearray()
        for i in ids:
            i = int(i)
            if i in self._by_id:
                out += self._by_id[i].encode("utf-8")
                continue
            for c in self._inverse.get(i, ""):
                out.append(self._byte_dec.get(c, 0))
        return out.decode("utf-8", errors="replace")

    def _encode_text(self, s: str) -> list[int]:
        ids: list[int] = []
        for word in self._split(s):
            ids.extend(self._bpe("".join(self._byte_enc[b] for b in word.encode("utf-8"))))
        return ids

    def _bpe(self, word: str) -> list[int]:
        """Merges the lowest-ranked adjacent pair (the leftmost among equals)
        until none is in the merges; parts missing from the vocabulary are
        dropped (tokenizer.go:280-309)."""
        hit = self._cache.get(word)
        if hit is not None:
            return hit
        parts = list(word)
        while len(parts) > 1:
            best, best_rank = -1, None
            for i in range(len(parts) - 1):
                r = self._ranks.get((parts[i], parts[i + 1]))
                if r is not None and (best_rank is None or r < best_rank):
                    best, best_rank = i, r
            if best < 0:
                break
            parts[best:best + 2] = [parts[best] + parts[best + 1]]
        ids = [self._vocab[p] for p in parts if p in self._vocab]
        self._cache[word] = ids
        return ids

    def _split(self, s: str) -> list[str]:
        """The pre-tokenization pattern as a scanner: at each position the
        pattern's alternatives in order (tokenizer.go:313-440)."""
        cfg, rs, out, i, n = self._split_cfg, s, [], 0, len(s)
        while i < n:
            if rs[i] == "'" and i + 1 < n:
                k = _match_contraction(rs[i:], cfg.ci_contractions)
                if k:
                    out.append(rs[i:i + k])
                    i += k
                    continue
            start = j = i
            # letters, after " ?" (GPT-2) or "[^\r\n\p{L}\p{N}]?" (cl100k)
            pfx = j
            if cfg.letter_prefix:
                c = rs[j]
                if not _is_letter(c) and not _is_number(c) and c not in "\r\n" and j + 1 < n and _is_letter(rs[j + 1]):
                    pfx = j + 1
            elif rs[j] == " " and j + 1 < n and _is_letter(rs[j + 1]):
                pfx = j + 1
            if pfx < n and _is_letter(rs[pfx]):
                j = pfx
                while j < n and _is_letter(rs[j]):
                    j += 1
                out.append(rs[start:j])
                i = j
                continue
            # numbers: " ?\p{N}+" (GPT-2) or "\p{N}{1,max}" (cl100k)
            if cfg.max_digits > 0:
                if _is_number(rs[j]):
                    while j < n and j - start < cfg.max_digits and _is_number(rs[j]):
                        j += 1
                    out.append(rs[start:j])
                    i = j
                    continue
            else:
                d = j
                if rs[d] == " " and d + 1 < n and _is_number(rs[d + 1]):
                    d += 1
                if d < n and _is_number(rs[d]):
                    j = d
                    while j < n and _is_number(rs[j]):
                        j += 1
                    out.append(rs[start:j])
                    i = j
                    continue
            # punctuation: " ?[^\s\p{L}\p{N}]+", then "[\r\n]*" (cl100k)
            p = j
            if rs[p] == " " and p + 1 < n and _is_punct(rs[p + 1]):
                p += 1
            if p < n and _is_punct(rs[p]):
                j = p
                while j < n and _is_punct(rs[j]):
                    j += 1
                if cfg.newline_runs:
                    while j < n and rs[j] in "\r\n":
                        j += 1
                out.append(rs[start:j])
                i = j
                continue
            # a white-space run [start, j)
            while j < n and _is_space(rs[j]):
                j += 1
            if cfg.newline_runs:  # "\s*[\r\n]+": through the run's last newline
                last = -1
                for k in range(start, j):
                    if rs[k] in "\r\n":
                        last = k
                if last >= 0:
                    out.append(rs[start:last + 1])
                    i = last + 1
                    continue
            # "\s+(?!\S)" then "\s+": the run's last character stays for what follows
            if j < n and j - start > 1:
                j -= 1
            if j == start:
                j += 1
            out.append(rs[start:j])
            i = j
        return out


def _match_contraction(rest: str, ci: bool) -> int:
    low = rest.lower() if ci else rest
    for c in _CONTRACTIONS:
        if low.startswith(c):
            return len(c)
    return 0


def Parse(raw) -> Tokenizer:
    """A Tokenizer from tokenizer.json bytes or text (tokenizer.go:86-150)."""
    try:
        f = json.loads(raw)
    except (ValueError, TypeError) as e:
        raise ValueError(f"tokenizer: parsing json: {e}") from None
    norm = f.get("normalizer")
    if norm is not None and not (isinstance(norm, dict) and norm.get("type") == "NFC"):
        raise ValueError(f"tokenizer: unsupported normalizer {json.dumps(norm)}")
    model = f.get("model") or {}
    if model.get("type", "") not in ("", "BPE"):
        raise ValueError(f"tokenizer: unsupported model type {model.get('type')!r}")
    vocab = model.get("vocab") or {}
    if not vocab:
        raise ValueError("tokenizer: empty vocab")
    split = _detect_split(f.get("pre_tokenizer"))
    ranks = {}
    for rank, m in enumerate(model.get("merges") or []):
        if isinstance(m, str):
            parts = m.split(" ", 1)
            if len(parts) != 2:
                raise ValueError(f"tokenizer: bad merge {m!r}")
            ranks[(parts[0], parts[1])] = rank
        else:
            a, b = m
            ranks[(a, b)] = rank
    # an empty added token would match everywhere (the Go loop never ends on it): left out
    specials = [(t["content"], int(t["id"])) for t in f.get("added_tokens") or [] if t.get("content")]
    return Tokenizer(vocab, ranks, specials, split)


def Load(path: str) -> Tokenizer:
    """Reads a tokenizer.json file."""
    with open(path, "rb") as fh:
        return Parse(fh.read())
