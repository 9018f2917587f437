"""Byte-level BPE tokenizer for Qwen tokenizer.json files, and the Qwen3.5 chat template with thinking disabled.

The host-side mirror of the reference's engine/tokenizer.js:1-151 (the reference checks it against Hugging Face
`tokenizers`, tests/tokenizer_ref.py): NFC normalisation, the pre-tokenizer's split regex, the GPT-2 byte-to-unicode
map, merges applied by rank, added tokens recognised in the text (longest first), decoding back to bytes, one-token
display pieces and the chat template.  Text never reaches the GPU; prompts enter the engine as token ids.
"""
import json
import unicodedata

import regex

# the pre-tokenizer split used when a tokenizer.json names none (tokenizer.js:35)
DEFAULT_SPLIT = r"'s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+"


def _byte_map():
    """GPT-2's reversible byte <-> printable-character map: printable Latin-1 bytes map to themselves, the other 68
    bytes to U+0100 onwards in byte order."""
    keep = list(range(33, 127)) + list(range(161, 173)) + list(range(174, 256))
    chars = {b: chr(b) for b in keep}
    n = 0
    for b in range(256):
        if b not in chars:
            chars[b] = chr(256 + n)
            n += 1
    return [chars[b] for b in range(256)]


BYTE_TO_CHAR = _byte_map()
CHAR_TO_BYTE = {c: b for b, c in enumerate(BYTE_TO_CHAR)}


class Tokenizer:
    """tokenizer.json (a dict) -> encode / decode / piece / units / chat, as engine/tokenizer.js."""

    def __init__(self, spec):
        m = spec["model"]
        if m.get("type") != "BPE":
            raise ValueError("only BPE tokenizers are supported")
        self.vocab = dict(m["vocab"])
        self.ranks = {}
        for i, mg in enumerate(m["merges"]):
            key = tuple(mg) if isinstance(mg, list) else tuple(mg.split(" ", 1))
            self.ranks.setdefault(key, i)
        size = max([*self.vocab.values(), *[a["id"] for a in spec.get("added_tokens", [])]], default=-1) + 1
        self.id_to_tok = [None] * size
        for t, i in self.vocab.items():
            self.id_to_tok[i] = t
        self.special = {}
        for a in spec.get("added_tokens", []):
            self.special[a["content"]] = a["id"]
            self.id_to_tok[a["id"]] = a["content"]
        self.special_ids = {a["id"] for a in spec.get("added_tokens", []) if a.get("special")}
        pattern = None
        pre = spec.get("pre_tokenizer") or {}
        for p in pre.get("pretokenizers", [pre]):
            if p.get("type") == "Split":
                pattern = (p.get("pattern") or {}).get("Regex")
                break
        self.split = regex.compile(pattern or DEFAULT_SPLIT)
        keys = sorted(self.special, key=len, reverse=True)
        self.special_re = regex.compile("(" + "|".join(regex.escape(k) for k in keys) + ")") if keys else None
        self.cache = {}
        self.size = len(self.id_to_tok)

    @classmethod
    def from_file(cls, path):
        with open(path, encoding="utf-8") as f:
            return cls(json.load(f))

    def _bpe(self, word):
        hit = self.cache.get(word)
        if hit is not None:
            return hit
        parts = list(word)
        while len(parts) > 1:
            best, at = None, -1
            for i in range(len(parts) - 1):
                r = self.ranks.get((parts[i], parts[i + 1]))
                if r is not None and (best is None or r < best):
                    best, at = r, i
            if at < 0:
                break
            pair = (parts[at], parts[at + 1])
            nxt, i = [], 0
            while i < len(parts):  # merge every occurrence of the best pair, left to right
                if i < len(parts) - 1 and (parts[i], parts[i + 1]) == pair:
                    nxt.append(parts[i] + parts[i + 1])
                    i += 2
                else:
                    nxt.append(parts[i])
                    i += 1
            parts = nxt
        ids = [self.vocab[p] for p in parts]
        if len(self.cache) > 50000:
            self.cache.clear()
        self.cache[word] = ids
        return ids

    def encode(self, text, special=True):
        """text -> ids; added tokens (e.g. <|im_start|>) in the text are recognised when `special`."""
        out = []
        pieces = self.special_re.split(text) if (special and self.special_re) else [text]
        for piece in pieces:
            if not piece:
                continue
            if special and piece in self.special:
                out.append(self.special[piece])
                continue
            norm = unicodedata.normalize("NFC", piece)
            for m in self.split.finditer(norm):
                w = "".join(BYTE_TO_CHAR[b] for b in m.group(0).encode("utf-8"))
                out.extend(self._bpe(w))
        return out

    def bytes(self, ids, skip_special=True):
        """ids -> the bytes of their text (special tokens included unless skip_special)."""
        out = bytearray()
        for i in ids:
            if skip_special and i in self.special_ids:
                continue
            t = self.id_to_tok[i] if 0 <= i < len(self.id_to_tok) else None
            if t is None:
                continue
            if t in self.special:
                out += t.encode("utf-8")
                continue
            for ch in t:
                b = CHAR_TO_BYTE.get(ch)
                if b is not None:
                    out.append(b)
        return bytes(out)

    def decode(self, ids, skip_special=True):
        return self.bytes(ids, skip_special).decode("utf-8", errors="replace")

    def piece(self, i):
        """Display string of one token; the bytes of a split character show as <hex>."""
        b = self.bytes([i], False)
        s = b.decode("utf-8", errors="replace")
        return "".join(f"<{x:02x}>" for x in b) if "�" in s else s

    def units(self, ids):
        """Token ids grouped into displayable units: the byte pieces of one multi-byte character join the token that
        completes it.  [{"text", "idx": [token indices]}] (tokenizer.js:107-130, emoji glue included)."""
        units, pending, prev, allids = [], [], "", []
        for i, t in enumerate(ids):
            allids.append(t)
            pending.append(i)
            full = self.decode(allids, False)
            if full.endswith("�") and i < len(ids) - 1:
                continue
            text = full[len(prev):] if full.startswith(prev) else self.decode([ids[j] for j in pending], False)
            units.append({"text": text, "idx": pending})
            prev, pending = full, []
        glue = regex.compile("^[\u200d\ufe0f\ufe0e\u20e3\U0001F3FB-\U0001F3FF]")
        ri_start = regex.compile("^[\U0001F1E6-\U0001F1FF]")

        def odd_ri(t):
            m = regex.search("[\U0001F1E6-\U0001F1FF]+$", t)
            return bool(m) and len(m.group(0)) % 2 == 1

        merged = []
        for u in units:
            last = merged[-1] if merged else None
            if last and u["text"] and (glue.match(u["text"]) or last["text"].endswith("\u200d") or
                                       (ri_start.match(u["text"]) and odd_ri(last["text"]))):
                last["text"] += u["text"]
                last["idx"] = last["idx"] + u["idx"]
            else:
                merged.append({"text": u["text"], "idx": list(u["idx"])})
        return merged

    def id(self, tok):
        return self.special.get(tok, self.vocab.get(tok))

    @staticmethod
    def chat(messages, generation=True):
        """Qwen3.5 chat template with thinking disabled (apply_chat_template(..., enable_thinking=False))."""
        s = "".join(f"<|im_start|>{m['role']}\n{m['content']}<|im_end|>\n" for m in messages)
        if generation:
            s += "<|im_start|>assistant\n<think>\n\n</think>\n\n"
        return s
