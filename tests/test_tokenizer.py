"""duo.tokenizer (the mirror of engine/tokenizer.js) against Hugging Face `tokenizers`, the library the reference
checks its tokenizer with (tests/tokenizer_ref.py).  No Qwen tokenizer.json is available offline, so the test trains
a small byte-level BPE of the same construction -- NFC normaliser, the Qwen split pattern, byte-level mapping, added
special tokens and the <think> markers -- on a short corpus written here, and compares ids, decoding, pieces and the
chat template on text that covers what the reference's own cases cover (accents in composed and decomposed form,
contractions in both cases, runs of spaces, tabs and CRLF, digits, code, CJK, RTL and Indic scripts, emoji with
joiners, flags and skin tones, special tokens inside the text)."""
import json
import unicodedata

import pytest

tokenizers = pytest.importorskip("tokenizers")

QWEN_SPLIT = (r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+"
              r"|\s+(?!\S)|\s+")
SPECIAL = ["<|endoftext|>", "<|im_start|>", "<|im_end|>"]

CORPUS = [
    "The river valley was settled by farmers, and later by traders who crossed the hills every spring.",
    "She said it's fine; they'll come back tomorrow, won't they? I'd rather we'd waited.",
    "Numbers like 42, 2026 and 3.14159 appear in tables; so do prices such as $19.99 and 7%.",
    "def area(r):\n    return 3.14159 * r * r\n\nfor i in range(10):\n    print(i, area(i))\n",
    "Café au lait, naïve façade, jalapeño, smörgåsbord, crème brûlée and the Zürich tram.",
    "東京は日本の首都です。今日は天気がいいので散歩に行きます。我们明天去图书馆看书。",
    "Привет, как дела? Всё хорошо. مرحبا كيف حالك نمستे दोस्त 안녕하세요 반갑습니다",
    "Emoji: 🙂 😀 👍🏽 👩‍💻 🇫🇷 🇯🇵 ❤️ 1️⃣ and symbols ½ ¾ → ← ✓ … “quotes” ‘single’",
    "   leading spaces, tabs\tinside, trailing   \r\nnew lines\n\n\nand more text after blank lines",
] * 6

CASES = [
    "Hello there, a café and a naïve plan: 7 items for 12 dollars.",
    "Café and naïve written with combining accents",
    "It's OK. IT'S OK. They'RE here, we'LL see, he'D go, I'M sure, you'VE won.",
    "  two leading spaces\n\n\ttab line\r\nwindows line   three trailing   ",
    "for k in range(3):\n    x = k * 2  # comment\n    print(f'{x:03d}')\n",
    "Mixed: 今日は晴れ 我们走吧 Здравствуйте שלום नमस्ते 안녕",
    "emoji 👩‍👩‍👧‍👦 family, 🇫🇷🇯🇵 flags, 👍🏽 tone, 1️⃣ keycap",
    "<|im_start|>user\nHow are you?<|im_end|>\n<|im_start|>assistant\n<think>\n\n</think>\n\nFine.",
    "1234567890 3.14159e-10 x=1&y=2 a.b@c.de (approx.) !!!??? ......",
    "",
]


@pytest.fixture(scope="module")
def pair():
    from tokenizers import Regex, Tokenizer as HF, decoders, models, normalizers, pre_tokenizers, trainers
    from duo.tokenizer import Tokenizer
    hf = HF(models.BPE())
    hf.normalizer = normalizers.NFC()
    hf.pre_tokenizer = pre_tokenizers.Sequence([
        pre_tokenizers.Split(Regex(QWEN_SPLIT), behavior="isolated", invert=False),
        pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    hf.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=900, special_tokens=SPECIAL,
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet(), show_progress=False)
    hf.train_from_iterator(CORPUS, trainer)
    hf.add_tokens(["<think>", "</think>"])  # added, not special (decoded like text)
    spec = json.loads(hf.to_str())
    return hf, Tokenizer(spec)


def test_encode_matches_tokenizers(pair):
    hf, tok = pair
    for text in CASES:
        assert tok.encode(text) == hf.encode(text).ids, text


def test_decode_round_trip_and_special_tokens(pair):
    hf, tok = pair
    for text in CASES:
        ids = tok.encode(text)
        assert tok.decode(ids, skip_special=False) == unicodedata.normalize("NFC", text)
        assert tok.decode(ids) == hf.decode(ids, skip_special_tokens=True)
    ids = tok.encode("<|im_start|>user\nhi<|im_end|>")
    assert ids[0] == tok.id("<|im_start|>") and ids[-1] == tok.id("<|im_end|>")
    assert tok.encode("<|im_start|>", special=False) != [tok.id("<|im_start|>")]  # plain text when not special


def test_pieces_and_units(pair):
    _, tok = pair
    ids = tok.encode("é日🙂")
    for i in ids:
        p = tok.piece(i)
        assert p and ("<" in p or "�" not in p)
    units = tok.units(tok.encode("a 👩‍💻 b 🇫🇷 c 👍🏽"))
    texts = [u["text"] for u in units]
    assert "".join(texts) == "a 👩‍💻 b 🇫🇷 c 👍🏽"
    assert any("👩‍💻" in t for t in texts)          # a joiner sequence stays one unit
    assert any("🇫🇷" in t for t in texts)                 # a flag (two regional indicators) stays one unit
    assert any("👍🏽" in t for t in texts)                 # a skin tone joins its emoji
    assert sorted(i for u in units for i in u["idx"]) == list(range(len(tok.encode("a 👩‍💻 b 🇫🇷 c 👍🏽"))))


def test_chat_template():
    from duo.tokenizer import Tokenizer
    s = Tokenizer.chat([{"role": "system", "content": "Be brief."}, {"role": "user", "content": "Hi"}])
    assert s == ("<|im_start|>system\nBe brief.<|im_end|>\n<|im_start|>user\nHi<|im_end|>\n"
                 "<|im_start|>assistant\n<think>\n\n</think>\n\n")
    assert Tokenizer.chat([{"role": "user", "content": "x"}], generation=False) == "<|im_start|>user\nx<|im_end|>\n"
