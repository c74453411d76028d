"""Text corpora -> a prepared byte-token file the loaders read.

The reference reads Hugging Face corpora (parquet / jsonl shards) and prepared token
chunks (burn_dragon_language/src/dataset/{huggingface,prepared_chunks}.rs). Here a
corpus directory or file of ``.jsonl`` (one JSON object per line, text under
``text_field``), ``.parquet`` (a ``text_field`` column, read with pyarrow) or ``.txt``
documents is tokenised once — UTF-8 bytes, documents separated by ``separator`` — into
``<cache_dir>/<name>.bin`` (uint8, the byte vocabulary of the BDH configurations), with
a ``.json`` manifest of the source files, sizes and modification times. A matching
manifest makes later runs reuse the file. The training loop then reads windows of it
(``dataset.type = "file"`` semantics: memory-mapped, train / valid split by ratio).
"""

from __future__ import annotations

import hashlib
import json
import os

import numpy as np


def _files(path: str) -> list[str]:
    if os.path.isfile(path):
        return [path]
    out = []
    for root, _, names in os.walk(path):
        for n in sorted(names):
            if n.endswith((".jsonl", ".parquet", ".txt")):
                out.append(os.path.join(root, n))
    return sorted(out)


def _documents(f: str, text_field: str):
    if f.endswith(".jsonl"):
        with open(f, encoding="utf-8") as fh:
            for line in fh:
                line = line.strip()
                if line:
                    t = json.loads(line).get(text_field)
                    if isinstance(t, str):
                        yield t
    elif f.endswith(".parquet"):
        import pyarrow.parquet as pq

        for batch in pq.ParquetFile(f).iter_batches(columns=[text_field]):
            for t in batch.column(0).to_pylist():
                if isinstance(t, str):
                    yield t
    else:
        with open(f, encoding="utf-8", errors="replace") as fh:
            yield fh.read()


def prepare_corpus(path: str, cache_dir: str, text_field: str = "text", separator: bytes = b"\n\n",
                   tokenizer: str | None = None) -> str:
    """Tokenise the corpus at ``path`` into a token file; returns its path. Without a
    ``tokenizer`` (a ``tokenizer.json``) the tokens are the UTF-8 bytes (uint8); with a
    BPE tokenizer they are its ids (uint16, vocabulary <= 65536). The manifest records
    ``token_bytes``."""
    files = _files(path)
    if not files:
        raise FileNotFoundError(f"no .jsonl / .parquet / .txt files under {path}")
    sig = [[f, os.path.getsize(f), int(os.path.getmtime(f))] for f in files]
    tok = None
    if tokenizer:
        from ..utils.tokenizer import load_tokenizer

        tok = load_tokenizer(tokenizer)
        if tok.vocab_size > 65536:
            raise ValueError("token files hold uint16 ids: vocabulary must be <= 65536")
        sig.append([tokenizer, os.path.getsize(tokenizer), int(os.path.getmtime(tokenizer))])
    key = hashlib.sha256(json.dumps([sig, text_field, separator.hex()]).encode()).hexdigest()[:16]
    os.makedirs(cache_dir, exist_ok=True)
    out = os.path.join(cache_dir, f"corpus-{key}.bin")
    man = out[:-4] + ".json"
    if os.path.exists(out) and os.path.exists(man):
        return out
    tmp = out + ".tmp"
    n_docs = 0
    with open(tmp, "wb") as fh:
        for f in files:
            for doc in _documents(f, text_field):
                if tok is None:
                    if n_docs:
                        fh.write(separator)
                    fh.write(doc.encode("utf-8"))
                else:
                    ids = tok.encode(doc)
                    if n_docs:
                        ids = tok.encode(separator.decode()) + ids
                    fh.write(np.asarray(ids, dtype="<u2").tobytes())
                n_docs += 1
    os.replace(tmp, out)
    with open(man, "w") as fh:
        json.dump({"sources": sig, "text_field": text_field, "documents": n_docs,
                   "bytes": os.path.getsize(out), "token_bytes": 1 if tok is None else 2,
                   "vocab": "bytes" if tok is None else tok.vocab_size}, fh, indent=2)
    return out


def token_bytes(path: str) -> int:
    """1 or 2: from the prepared file's manifest (1 when there is none: a plain byte file)."""
    man = path[:-4] + ".json" if path.endswith(".bin") else None
    if man and os.path.exists(man):
        return int(json.load(open(man)).get("token_bytes", 1))
    return 1


def corpus_bytes(path: str) -> np.ndarray:
    return np.memmap(path, dtype=np.uint8, mode="r")
