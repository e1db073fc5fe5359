"""The byte-level BPE tokenizer (qwen0.6b_b200/tokenizer.py) against the
Hugging Face ``tokenizers`` library that upstream's AutoTokenizer runs
(Model/Qwen06B_architecture.py:125, :345, :379-382).

The Qwen3 tokenizer files are not available offline, so the pin is a
tokenizer of the same pipeline trained here by ``tokenizers`` itself on seeded
synthetic text: NFC normalizer, Split by the Qwen2-family pre-tokenizer regex
(behaviour Isolated), ByteLevel without its own regex, BPE, ByteLevel decoder,
with chat special tokens.  Encodings and decodings must be identical, id for
id and character for character.
"""
import json
import random

import pytest

tokenizers = pytest.importorskip("tokenizers")

from tokenizer import QwenTokenizer, bytes_to_unicode  # noqa: E402

# The pre-tokenizer regex of the Qwen2/Qwen3 tokenizer family.
PATTERN = (r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*"
           r"|\s*[\r\n]+|\s+(?!\S)|\s+")
SPECIALS = ["<|endoftext|>", "<|im_start|>", "<|im_end|>"]

_ALPHABETS = [
    "abcdefghijklmnopqrstuvwxyz", "ABCDEFGHIJKLMNOPQRSTUVWXYZ", "0123456789",
    "äöüßéèêàçñ", "абвгдежзийклмнопрст", "的一是不了人我在有他这中大来上国",
    "αβγδεζηθικλμ", ".,;:!?'\"()[]{}-_/\\@#$%^&*+=<>|~`", "😀🚀✨🎉",
]


def _word(rng):
    alpha = rng.choice(_ALPHABETS)
    return "".join(rng.choice(alpha) for _ in range(rng.randint(1, 9)))


def _text(rng, n_words):
    seps = [" ", " ", " ", "  ", "\n", "\n\n", "\t", " \n ", "'s ", "'ll ", "'RE "]
    return "".join(_word(rng) + rng.choice(seps) for _ in range(n_words))


@pytest.fixture(scope="module", params=[False, True], ids=["merges", "ignore_merges"])
def pair(request, tmp_path_factory):
    from tokenizers import Regex, Tokenizer, decoders, models, normalizers, pre_tokenizers, trainers
    rng = random.Random(1234)
    corpus = [_text(rng, 40) for _ in range(400)]
    tok = Tokenizer(models.BPE(ignore_merges=request.param))
    tok.normalizer = normalizers.NFC()
    tok.pre_tokenizer = pre_tokenizers.Sequence([
        pre_tokenizers.Split(Regex(PATTERN), behavior="isolated", invert=False),
        pre_tokenizers.ByteLevel(add_prefix_space=False, trim_offsets=False, use_regex=False),
    ])
    tok.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=1500, initial_alphabet=pre_tokenizers.ByteLevel.alphabet(),
                                  special_tokens=SPECIALS, show_progress=False)
    tok.train_from_iterator(corpus, trainer)
    d = tmp_path_factory.mktemp("tok")
    tok.save(str(d / "tokenizer.json"))
    (d / "tokenizer_config.json").write_text(json.dumps(
        {"eos_token": "<|im_end|>", "pad_token": "<|endoftext|>", "bos_token": None,
         "clean_up_tokenization_spaces": False}))
    return tok, QwenTokenizer.from_dir(str(d))


def test_byte_alphabet_is_a_bijection():
    t = bytes_to_unicode()
    assert len(t) == 256 and len(set(t.values())) == 256
    assert all(c.isprintable() and not c.isspace() for c in t.values())
    assert t[ord("A")] == "A" and t[ord(" ")] == chr(0x120)


def test_encode_matches_tokenizers(pair):
    ref, ours = pair
    rng = random.Random(99)
    cases = [_text(rng, rng.randint(1, 30)) for _ in range(300)]
    cases += ["", " ", "   ", "\n", "\r\n\r\n", "a", "A's", "I'M here", "x  y", "tab\tsep", "12345678",
              "é", "Ａｂｃ", "emoji 🚀🚀 run", "mixed中文and English", "trailing space ",
              " nbsp", "\x00\x01ctrl", "ﬁ ligature"]
    for s in cases:
        assert ours.encode(s) == ref.encode(s).ids, repr(s)


def test_special_tokens_inside_text(pair):
    ref, ours = pair
    s = ("<|im_start|>system\nYou are a helpful assistant.<|im_end|>\n<|im_start|>user\nhi<|im_end|>"
         "\n<|im_start|>assistant\n<|im_end|><|endoftext|>x<|im_end|>")
    assert ours.encode(s) == ref.encode(s).ids
    assert ours.encode(s, add_special_tokens=False) == ref.encode(s, add_special_tokens=False).ids


def test_decode_matches_tokenizers(pair):
    ref, ours = pair
    rng = random.Random(5)
    for _ in range(200):
        s = _text(rng, rng.randint(1, 20)) + rng.choice(["", "<|im_end|>", "<|endoftext|> tail"])
        ids = ref.encode(s).ids
        assert ours.decode(ids) == ref.decode(ids, skip_special_tokens=False)
        assert ours.decode(ids, skip_special_tokens=True) == ref.decode(ids, skip_special_tokens=True)
    # Arbitrary id sequences, including ones that cut UTF-8 sequences apart.
    n = ref.get_vocab_size()
    for _ in range(200):
        ids = [rng.randrange(n) for _ in range(rng.randint(1, 12))]
        assert ours.decode(ids) == ref.decode(ids, skip_special_tokens=False)


def test_special_token_ids_and_call_form(pair):
    ref, ours = pair
    assert ours.eos_token_id == ref.token_to_id("<|im_end|>")
    assert ours.pad_token_id == ref.token_to_id("<|endoftext|>")
    assert ours.bos_token_id is None
    enc = ours("hello world", return_tensors="pt")
    assert enc.input_ids.shape == (1, len(ref.encode("hello world").ids))
    assert enc.input_ids[0].tolist() == ref.encode("hello world").ids
    assert len(ours) == ref.get_vocab_size()


def test_unsupported_pipelines_raise():
    base = {"model": {"type": "BPE", "vocab": {"a": 0}, "merges": []},
            "pre_tokenizer": {"type": "ByteLevel", "add_prefix_space": False, "use_regex": True}}
    QwenTokenizer(base)
    with pytest.raises(NotImplementedError):
        QwenTokenizer({**base, "model": {"type": "WordPiece", "vocab": {}}})
    with pytest.raises(NotImplementedError):
        QwenTokenizer({**base, "normalizer": {"type": "Lowercase"}})
