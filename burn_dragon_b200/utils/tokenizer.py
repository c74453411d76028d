"""Tokenizers: the byte tokenizer (vocab 256, the BDH configurations) and a byte-level
BPE with GPT-4-style pre-splitting (burn_dragon_tokenizer/src/lib.rs).

BPE training: split text with the GPT-4 pattern, count words, then repeatedly merge the
most frequent adjacent pair (ties broken by the smaller pair) into a new id, updating
pair counts incrementally per affected word; encoding applies merges by rank inside
each pre-split chunk. ``tokenizer.json`` stores ``{"type": "bpe", "pattern", "merges"}``.
"""

from __future__ import annotations

import heapq
import json
from collections import Counter, defaultdict

import regex

GPT4_PATTERN = (r"'(?i:[sdmt]|ll|ve|re)|[^\r\n\p{L}\p{N}]?+\p{L}+|\p{N}{1,3}| ?[^\s\p{L}\p{N}]++[\r\n]*"
                r"|\s*[\r\n]|\s+(?!\S)|\s+")


class ByteTokenizer:
    vocab_size = 256

    def encode(self, text: str) -> list[int]:
        return list(text.encode("utf-8"))

    def decode(self, ids) -> str:
        return bytes(int(i) & 0xFF for i in ids).decode("utf-8", errors="replace")

    def to_json(self) -> dict:
        return {"type": "byte", "vocab_size": 256}


class BPETokenizer:
    def __init__(self, merges: dict[tuple[int, int], int] | None = None, pattern: str = GPT4_PATTERN):
        self.merges = dict(merges or {})
        self.pattern = pattern
        self._re = regex.compile(pattern)

    @property
    def vocab_size(self) -> int:
        return 256 + len(self.merges)

    # ---------------------------------------------------------------- training
    def train(self, texts, vocab_size: int) -> "BPETokenizer":
        if vocab_size < 256:
            raise ValueError("vocab_size must be >= 256")
        words: Counter = Counter()
        for t in texts:
            for w in self._re.findall(t):
                words[w.encode("utf-8")] += 1
        seqs = [list(w) for w in words]
        freq = list(words.values())
        pair_count: Counter = Counter()
        where: dict[tuple[int, int], set[int]] = defaultdict(set)
        for i, s in enumerate(seqs):
            for a, b in zip(s, s[1:]):
                pair_count[(a, b)] += freq[i]
                where[(a, b)].add(i)
        heap = [(-c, p) for p, c in pair_count.items()]
        heapq.heapify(heap)
        merges: dict[tuple[int, int], int] = {}
        next_id = 256
        while next_id < vocab_size and heap:
            negc, pair = heapq.heappop(heap)
            if pair_count.get(pair, 0) != -negc or -negc <= 0:
                continue  # stale heap entry
            merges[pair] = next_id
            for i in list(where[pair]):
                s = seqs[i]
                f = freq[i]
                for a, b in zip(s, s[1:]):
                    pair_count[(a, b)] -= f
                out, k = [], 0
                while k < len(s):
                    if k + 1 < len(s) and s[k] == pair[0] and s[k + 1] == pair[1]:
                        out.append(next_id)
                        k += 2
                    else:
                        out.append(s[k])
                        k += 1
                seqs[i] = out
                for a, b in zip(out, out[1:]):
                    pair_count[(a, b)] += f
                    where[(a, b)].add(i)
                    heapq.heappush(heap, (-pair_count[(a, b)], (a, b)))
            del where[pair]
            next_id += 1
        self.merges = merges
        return self

    # ---------------------------------------------------------------- coding
    def _encode_chunk(self, ids: list[int]) -> list[int]:
        while len(ids) >= 2:
            best = min(((self.merges.get(p, 1 << 60), j) for j, p in enumerate(zip(ids, ids[1:]))))
            rank, j = best
            if rank == 1 << 60:
                break
            ids = ids[:j] + [rank] + ids[j + 2:]
        return ids

    def encode(self, text: str) -> list[int]:
        out: list[int] = []
        for w in self._re.findall(text):
            out.extend(self._encode_chunk(list(w.encode("utf-8"))))
        return out

    def decode(self, ids) -> str:
        table = {i: bytes([i]) for i in range(256)}
        for (a, b), i in sorted(self.merges.items(), key=lambda kv: kv[1]):
            table[i] = table[a] + table[b]
        return b"".join(table[int(i)] for i in ids).decode("utf-8", errors="replace")

    def to_json(self) -> dict:
        return {"type": "bpe", "pattern": self.pattern,
                "merges": [[a, b, i] for (a, b), i in sorted(self.merges.items(), key=lambda kv: kv[1])]}

    @staticmethod
    def from_json(d: dict) -> "BPETokenizer":
        return BPETokenizer({(a, b): i for a, b, i in d["merges"]}, d.get("pattern", GPT4_PATTERN))


def load_tokenizer(path_or_dict) -> ByteTokenizer | BPETokenizer:
    d = json.load(open(path_or_dict)) if isinstance(path_or_dict, str) else path_or_dict
    return BPETokenizer.from_json(d) if d.get("type") == "bpe" else ByteTokenizer()
