"""Native byte-level BPE tokenizer against the HF `tokenizers` library.

A small BPE is trained with the Qwen2 pre-tokenizer (split pattern + byte
level, NFC normalizer, chat special tokens), saved as tokenizer.json, and
loaded both ways; encode and decode must agree on text chosen to exercise
every alternative of the split pattern.
"""

import json

import pytest

tokenizers = pytest.importorskip("tokenizers")

from quail_b200.api.tokenizer import (QWEN2_SPLIT, HFTokenizer, NativeBpeTokenizer, _native_compatible,  # noqa: E402
                                      load_tokenizer)

CORPUS = [
    "The quick brown fox jumps over the lazy dog. It's 2024, isn't it? We'll see; they'd know.",
    "Résumé naïve café — déjà vu. Ñandú, Ærøskøbing, straße, ΑΒΓ δέλτα, Москва, 東京都, 서울.",
    "def f(x):\n    return x ** 2  # square\n\n\nclass A:\n\tpass\r\n",
    "Numbers: 1234567890 ½ Ⅻ ٣٤٥ and symbols !!! ??? ... --- *** ((( ))) {{}} <<>>",
    "Emoji 😀🎉👍🏽 and tabs\t\tand   spaces    and\n\nnewlines\r\n\r\nend",
    "I'M HERE, YOU'RE THERE, THEY'VE GONE, SHE'D SAY, HE'LL GO, IT'S OK, DON'T.",
] * 20

SPECIAL = ["<|endoftext|>", "<|im_start|>", "<|im_end|>", "<think>", "</think>"]

CASES = [
    "",
    "hello",
    " hello world",
    "  two spaces before",
    "trailing spaces   ",
    "tab\tseparated\tvalues",
    "It's a dog's life; we're sure they've gone, I'm told you'll see, he'd say.",
    "SHOUTING: IT'S DON'T WON'T 'S 'T 'RE",
    "'quote' ''double'' 'x",
    "numbers 12345 and 3.14159 and -42 and 1,000,000",
    "mixed123abc456",
    "Unicode: Résumé naïve café déjà Ærøskøbing straße Москва 東京都 서울",
    "Combining: e\u0301 a\u0308 (NFC folds these)",
    "emoji 😀 🎉👍🏽 done",
    "line one\nline two\n\n\nline five\r\nwindows\r\n",
    "   \n   leading whitespace then newline",
    "symbols !!! ??? ... --- *** ((( ))) {{}} <<>> @@@ ### $$$ %%%",
    " ?!punct with space\n\nand newlines after symbols!!\n\n",
    "code:\n    def f(x):\n        return x ** 2\n",
    "<|im_start|>user\nIs this relevant?<|im_end|>\n<|im_start|>assistant\n<think>\n\n</think>\n\nYes",
    "special<|endoftext|>glued<|im_end|><|im_end|>",
    "partial <|im_sta and <|im_end",
    "nbsp\u00a0here and ideographic\u3000space and em\u2003space",
    "Ⅻ½٣٤٥ numerals",
    "x" * 300,
    "\u00ad soft hyphen and \u200b zero width",
]


@pytest.fixture(scope="module")
def tok_path(tmp_path_factory):
    from tokenizers import Regex, Tokenizer, decoders, models, normalizers, pre_tokenizers, trainers
    tok = Tokenizer(models.BPE())
    tok.normalizer = normalizers.NFC()
    tok.pre_tokenizer = pre_tokenizers.Sequence([
        pre_tokenizers.Split(Regex(QWEN2_SPLIT), behavior="isolated", invert=False),
        pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False),
    ])
    tok.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=1200, special_tokens=SPECIAL,
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet(), show_progress=False)
    tok.train_from_iterator(CORPUS, trainer=trainer)
    d = tmp_path_factory.mktemp("tok")
    path = str(d / "tokenizer.json")
    tok.save(path)
    return path


def test_spec_is_native_compatible(tok_path):
    with open(tok_path, encoding="utf-8") as f:
        spec = json.load(f)
    assert _native_compatible(spec)
    assert isinstance(load_tokenizer(tok_path, 0), NativeBpeTokenizer)


@pytest.mark.parametrize("text", CASES)
def test_encode_decode_match_hf(tok_path, text):
    hf = HFTokenizer(tok_path)
    nat = NativeBpeTokenizer(tok_path)
    a = hf.encode(text).tolist()
    b = nat.encode(text).tolist()
    assert a == b, (text, a, b)
    assert nat.decode(b) == hf.decode(a)


def test_batch_and_corpus(tok_path):
    hf = HFTokenizer(tok_path)
    nat = NativeBpeTokenizer(tok_path)
    texts = CORPUS[:6] + CASES
    got = nat.encode_batch(texts)
    for t, g in zip(texts, got):
        assert g.tolist() == hf.encode(t).tolist()
    # the cache must not change results on repeat
    assert [g.tolist() for g in nat.encode_batch(texts)] == [g.tolist() for g in got]


def test_specials_and_ids(tok_path):
    nat = NativeBpeTokenizer(tok_path)
    hf = HFTokenizer(tok_path)
    for s in SPECIAL:
        assert nat.token_id(s) == hf.token_id(s)
    assert nat.token_id("definitely-not-a-token-xyz") is None
    assert set(nat.eos_ids) == set(hf.eos_ids)
    assert nat.vocab == hf.vocab
    assert nat.answer_ids(["Yes", "No", "Yes"]) == hf.answer_ids(["Yes", "No", "Yes"])


def test_other_pretokenizers_fall_back(tok_path):
    with open(tok_path, encoding="utf-8") as f:
        spec = json.load(f)
    spec["pre_tokenizer"] = {"type": "Whitespace"}
    assert not _native_compatible(spec)
    spec2 = json.loads(json.dumps(spec))
    spec2["model"]["type"] = "WordPiece"
    assert not _native_compatible(spec2)
