"""Restatement of the reference's BGE WordPiece tokenizer (src/tokenizer.cpp:9-160) and
its [CLS]/[SEP] framing (src/sentence_transformers_impl.cpp:17-22).

TEST INFRASTRUCTURE ONLY: the checker for the drop-in SentenceTransformer's tokenize()."""
from __future__ import annotations


class WordPiece:
    def __init__(self, vocab_lines: list[str]):
        self.vocab: dict[str, int] = {}
        for i, tok in enumerate(vocab_lines):
            self.vocab[tok] = i  # a repeated line keeps its last id, as a map assignment does
        self.unk = self.vocab["[UNK]"]

    @staticmethod
    def words(text: bytes) -> list[bytes]:
        """Byte-level split: ASCII whitespace (isspace) separates; a UTF-8 lead byte starts
        a one-character word; ASCII alnum accumulates lower-cased; other ASCII bytes stand
        alone; a stray or truncated byte becomes [UNK]."""
        out, cur, i = [], b"", 0
        space = b" \t\n\v\f\r"
        while i < len(text):
            c = text[i]
            if c in space:
                if cur:
                    out.append(cur)
                    cur = b""
                i += 1
                continue
            if c & 0x80:
                n = 2 if (c & 0xE0) == 0xC0 else 3 if (c & 0xF0) == 0xE0 else 4 if (c & 0xF8) == 0xF0 else 0
                if n == 0 or i + n > len(text):
                    out.append(b"[UNK]")
                    i += 1
                    continue
                if cur:
                    out.append(cur)
                    cur = b""
                out.append(text[i:i + n])
                i += n
                continue
            ch = bytes([c])
            if ch.isalnum():
                cur += ch.lower()
            else:
                if cur:
                    out.append(cur)
                    cur = b""
                out.append(ch)
            i += 1
        if cur:
            out.append(cur)
        return out

    def pieces(self, w: bytes) -> list[int]:
        key = w.decode("utf-8", errors="surrogateescape")
        if key in self.vocab:
            return [self.vocab[key]]
        found, start = [], 0
        while start < len(w):
            for end in range(len(w), start, -1):
                sub = (b"##" if start > 0 else b"") + w[start:end]
                k = sub.decode("utf-8", errors="surrogateescape")
                if k in self.vocab:
                    found.append(self.vocab[k])
                    start = end
                    break
            else:
                return [self.unk]
        return found

    def encode(self, text: str) -> list[int]:
        ids = [101]
        for w in self.words(text.encode("utf-8")):
            ids += self.pieces(w)
        return ids + [102]
