"""Byte-level BPE tokenizer read from a checkpoint's ``tokenizer.json``.

Replaces ``AutoTokenizer.from_pretrained`` in upstream ``load_weights``
(``Model/Qwen06B_architecture.py:125``) for the calls upstream makes:
``encode(prompt, add_special_tokens=True)`` (``:345``), ``eos_token_id``
(``:379``), ``decode(ids, skip_special_tokens=True)`` (``:382``) and
``tokenizer(text, return_tensors="pt").input_ids`` (``Model/benchmark.py:56``).

Qwen3 ships a Hugging Face ``tokenizers`` pipeline; this module restates the
published algorithm of each stage that pipeline uses and reads every table and
pattern from the file:

* added tokens (``added_tokens``): the text is first cut at every occurrence
  of an added token (longest match first; ``lstrip``/``rstrip`` absorb the
  adjacent whitespace); those pieces map straight to their ids;
* normalizer: Unicode NFC / NFD / NFKC / NFKD (or a sequence of them);
* pre-tokenizer: ``Split`` by the file's regex (behaviour ``Isolated``: every
  match and every non-matching gap is a piece), then ``ByteLevel``: each
  UTF-8 byte of a piece is mapped to one printable character (the GPT-2 byte
  table: printable Latin-1 bytes stand for themselves, the other 68 bytes are
  numbered from U+0100 upward);
* model: BPE with the merge ranks of ``merges`` — repeatedly join the
  adjacent pair of lowest rank (all its occurrences, left to right) until no
  pair has a rank; with ``ignore_merges`` a piece already in the vocabulary
  is one token;
* decoder: ``ByteLevel`` — the token strings' characters back to bytes, UTF-8
  decoded with U+FFFD for invalid sequences.

Special-token ids (eos, pad, bos) come from ``tokenizer_config.json``.
"""
from __future__ import annotations

import json
import os
import unicodedata

try:
    import regex as _re  # \p{L} / \p{N} classes, as the tokenizers' regex engine has them
except ImportError:  # pragma: no cover - the image ships regex
    _re = None


def bytes_to_unicode() -> dict[int, str]:
    """The byte-level alphabet: byte -> one printable character."""
    keep = list(range(ord("!"), ord("~") + 1)) + list(range(0xA1, 0xAC + 1)) + list(range(0xAE, 0xFF + 1))
    table, extra = {}, 0
    for b in range(256):
        if b in keep:
            table[b] = chr(b)
        else:
            table[b] = chr(256 + extra)
            extra += 1
    return table


_BYTE_ENC = bytes_to_unicode()
_BYTE_DEC = {c: b for b, c in _BYTE_ENC.items()}

# GPT-2's pre-tokenizer pattern, used by a ByteLevel pre-tokenizer with
# use_regex = true.
_GPT2_PATTERN = r"""'s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+"""


class _Encoding:
    def __init__(self, ids: list[int], return_tensors: str | None):
        if return_tensors == "pt":
            import torch
            self.input_ids = torch.tensor([ids], dtype=torch.long)
        elif return_tensors is None:
            self.input_ids = ids
        else:
            raise ValueError(f"return_tensors={return_tensors!r} is not supported")

    def __getitem__(self, key):
        return getattr(self, key)


class QwenTokenizer:
    """Encoder/decoder over one ``tokenizer.json`` (see the module docstring)."""

    def __init__(self, spec: dict, config: dict | None = None):
        if _re is None:
            raise RuntimeError("the 'regex' module is required for the pre-tokenizer patterns")
        config = config or {}
        model = spec.get("model") or {}
        if model.get("type", "BPE") != "BPE":
            raise NotImplementedError(f"tokenizer model {model.get('type')!r} (only BPE)")
        for k in ("continuing_subword_prefix", "end_of_word_suffix"):
            if model.get(k):
                raise NotImplementedError(f"BPE {k} is not supported")
        if model.get("dropout"):
            raise NotImplementedError("BPE dropout is not supported")
        self.vocab: dict[str, int] = dict(model["vocab"])
        self.ranks: dict[tuple[str, str], int] = {}
        for r, m in enumerate(model.get("merges", [])):
            a, b = m.split(" ", 1) if isinstance(m, str) else m
            self.ranks.setdefault((a, b), r)
        self.ignore_merges = bool(model.get("ignore_merges", False))
        self.byte_fallback = bool(model.get("byte_fallback", False))
        self.unk_token = model.get("unk_token")
        self.added: dict[str, dict] = {}
        for t in spec.get("added_tokens", []):
            self.added[t["content"]] = t
            self.vocab.setdefault(t["content"], t["id"])
        self.id_to_token = {i: t for t, i in self.vocab.items()}
        for t in spec.get("added_tokens", []):
            self.id_to_token[t["id"]] = t["content"]
        self.special_ids = {t["id"] for t in spec.get("added_tokens", []) if t.get("special")}
        self._normalizers = self._parse_normalizer(spec.get("normalizer"))
        self._pre = self._parse_pre_tokenizer(spec.get("pre_tokenizer"))
        self._post = self._parse_post_processor(spec.get("post_processor"))
        dec = spec.get("decoder")
        if dec is not None and dec.get("type") not in ("ByteLevel",):
            raise NotImplementedError(f"decoder {dec.get('type')!r} (only ByteLevel)")
        if self.added:
            alts = sorted(self.added, key=len, reverse=True)
            self._added_re = _re.compile("|".join(_re.escape(a) for a in alts))
        else:
            self._added_re = None
        self.clean_up_tokenization_spaces = bool(config.get("clean_up_tokenization_spaces", False))
        self.eos_token = self._token_str(config.get("eos_token"))
        self.pad_token = self._token_str(config.get("pad_token"))
        self.bos_token = self._token_str(config.get("bos_token"))
        self._cache: dict[str, list[int]] = {}

    # ------------------------------------------------------------ loading
    @classmethod
    def from_dir(cls, path: str) -> "QwenTokenizer":
        with open(os.path.join(path, "tokenizer.json"), encoding="utf-8") as f:
            spec = json.load(f)
        cfg_path = os.path.join(path, "tokenizer_config.json")
        config = {}
        if os.path.exists(cfg_path):
            with open(cfg_path, encoding="utf-8") as f:
                config = json.load(f)
        return cls(spec, config)

    @staticmethod
    def _token_str(v):
        if isinstance(v, dict):
            return v.get("content")
        return v

    @staticmethod
    def _parse_normalizer(n) -> list[str]:
        if n is None:
            return []
        kind = n.get("type")
        if kind == "Sequence":
            out = []
            for sub in n.get("normalizers", []):
                out += QwenTokenizer._parse_normalizer(sub)
            return out
        if kind in ("NFC", "NFD", "NFKC", "NFKD"):
            return [kind]
        raise NotImplementedError(f"normalizer {kind!r}")

    @staticmethod
    def _parse_pre_tokenizer(p) -> list[tuple]:
        if p is None:
            return []
        kind = p.get("type")
        if kind == "Sequence":
            out = []
            for sub in p.get("pretokenizers", []):
                out += QwenTokenizer._parse_pre_tokenizer(sub)
            return out
        if kind == "Split":
            pat = p["pattern"]
            src = pat["Regex"] if "Regex" in pat else _re.escape(pat["String"])
            if p.get("behavior", "Isolated") != "Isolated" or p.get("invert", False):
                raise NotImplementedError("Split behaviours other than Isolated (not inverted)")
            return [("split", _re.compile(src))]
        if kind == "ByteLevel":
            rx = _re.compile(_GPT2_PATTERN) if p.get("use_regex", True) else None
            return [("bytelevel", bool(p.get("add_prefix_space", False)), rx)]
        raise NotImplementedError(f"pre-tokenizer {kind!r}")

    @staticmethod
    def _parse_post_processor(p):
        if p is None or p.get("type") == "ByteLevel":
            return None
        if p.get("type") == "TemplateProcessing":
            return p
        raise NotImplementedError(f"post-processor {p.get('type')!r}")

    # ------------------------------------------------------------ encoding
    @property
    def eos_token_id(self) -> int | None:
        return self.vocab.get(self.eos_token) if self.eos_token is not None else None

    @property
    def pad_token_id(self) -> int | None:
        return self.vocab.get(self.pad_token) if self.pad_token is not None else None

    @property
    def bos_token_id(self) -> int | None:
        return self.vocab.get(self.bos_token) if self.bos_token is not None else None

    def __len__(self) -> int:
        return len(self.id_to_token)

    @property
    def vocab_size(self) -> int:
        return len(self.vocab)

    def convert_tokens_to_ids(self, tokens):
        if isinstance(tokens, str):
            return self.vocab.get(tokens)
        return [self.vocab.get(t) for t in tokens]

    def _split_added(self, text: str) -> list[tuple[str, bool]]:
        """(piece, is_added_token) in order."""
        if self._added_re is None or not text:
            return [(text, False)] if text else []
        out, pos = [], 0
        for m in self._added_re.finditer(text):
            tok = self.added[m.group(0)]
            start, end = m.start(), m.end()
            if start < pos:
                continue
            left = text[pos:start]
            if tok.get("lstrip"):
                left = left.rstrip()
            if left:
                out.append((left, False))
            out.append((m.group(0), True))
            pos = end
            if tok.get("rstrip"):
                while pos < len(text) and text[pos].isspace():
                    pos += 1
        if pos < len(text):
            out.append((text[pos:], False))
        return out

    def _pre_tokenize(self, text: str) -> list[str]:
        pieces = [text]
        byte_level = False
        for stage in self._pre:
            if stage[0] == "split":
                rx = stage[1]
                nxt = []
                for p in pieces:
                    pos = 0
                    for m in rx.finditer(p):
                        if m.start() > pos:
                            nxt.append(p[pos:m.start()])
                        if m.end() > m.start():
                            nxt.append(m.group(0))
                        pos = m.end()
                    if pos < len(p):
                        nxt.append(p[pos:])
                pieces = nxt
            else:
                _, prefix, rx = stage
                nxt = []
                for i, p in enumerate(pieces):
                    if prefix and i == 0 and not p.startswith(" "):
                        p = " " + p
                    sub = [m.group(0) for m in rx.finditer(p)] if rx is not None else [p]
                    nxt += ["".join(_BYTE_ENC[b] for b in s.encode("utf-8")) for s in sub]
                pieces = nxt
                byte_level = True
        if not byte_level:
            raise NotImplementedError("pre-tokenizer pipelines without a ByteLevel stage")
        return [p for p in pieces if p]

    def _bpe(self, word: str) -> list[int]:
        hit = self._cache.get(word)
        if hit is not None:
            return hit
        if self.ignore_merges and word in self.vocab:
            ids = [self.vocab[word]]
        else:
            syms = list(word)
            while len(syms) > 1:
                best, best_rank = None, None
                for i in range(len(syms) - 1):
                    r = self.ranks.get((syms[i], syms[i + 1]))
                    if r is not None and (best_rank is None or r < best_rank):
                        best, best_rank = (syms[i], syms[i + 1]), r
                if best is None:
                    break
                merged, i = [], 0
                while i < len(syms):
                    if i + 1 < len(syms) and (syms[i], syms[i + 1]) == best:
                        merged.append(syms[i] + syms[i + 1])
                        i += 2
                    else:
                        merged.append(syms[i])
                        i += 1
                syms = merged
            ids = []
            for s in syms:
                if s in self.vocab:
                    ids.append(self.vocab[s])
                elif self.unk_token is not None and self.unk_token in self.vocab:
                    ids.append(self.vocab[self.unk_token])
                else:
                    raise KeyError(f"symbol {s!r} is not in the vocabulary and there is no unk token")
        if len(self._cache) < 200_000:
            self._cache[word] = ids
        return ids

    def encode(self, text: str, add_special_tokens: bool = True) -> list[int]:
        ids: list[int] = []
        for piece, is_added in self._split_added(text):
            if is_added:
                ids.append(self.added[piece]["id"])
                continue
            for form in self._normalizers:
                piece = unicodedata.normalize(form, piece)
            for word in self._pre_tokenize(piece):
                ids += self._bpe(word)
        if add_special_tokens and self._post is not None:
            ids = self._apply_template(ids)
        return ids

    def _apply_template(self, ids: list[int]) -> list[int]:
        out = []
        specials = self._post.get("special_tokens", {})
        for item in self._post.get("single", []):
            if "SpecialToken" in item:
                out += specials[item["SpecialToken"]["id"]]["ids"]
            elif "Sequence" in item:
                out += ids
        return out

    def __call__(self, text: str, return_tensors: str | None = None, add_special_tokens: bool = True):
        return _Encoding(self.encode(text, add_special_tokens=add_special_tokens), return_tensors)

    # ------------------------------------------------------------ decoding
    def decode(self, ids, skip_special_tokens: bool = False) -> str:
        if hasattr(ids, "tolist"):
            ids = ids.tolist()
        if isinstance(ids, int):
            ids = [ids]
        raw = bytearray()
        for i in ids:
            i = int(i)
            if skip_special_tokens and i in self.special_ids:
                continue
            tok = self.id_to_token.get(i)
            if tok is None:
                continue
            if all(c in _BYTE_DEC for c in tok):
                raw += bytes(_BYTE_DEC[c] for c in tok)
            else:
                raw += tok.encode("utf-8")
        text = raw.decode("utf-8", errors="replace")
        if self.clean_up_tokenization_spaces:
            for a, b in ((" .", "."), (" ?", "?"), (" !", "!"), (" ,", ","), (" ' ", "'"), (" n't", "n't"),
                         (" 'm", "'m"), (" 's", "'s"), (" 've", "'ve"), (" 're", "'re")):
                text = text.replace(a, b)
        return text
