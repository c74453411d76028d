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


# ------------------------------------------------------------------ Hugging Face sources
# The reference pulls dataset repositories from the Hugging Face hub into a local cache and
# renders their records (burn_dragon_language/src/dataset/huggingface.rs, config schema
# schema.rs:37-96). This machine class trains without network access, so the source here
# is the hub's on-disk cache layout, filled beforehand by any hub client:
#   <hub cache>/datasets--<org>--<name>/refs/<revision>   (the snapshot id)
#   <hub cache>/datasets--<org>--<name>/snapshots/<id>/<repo files>
# The hub cache is ``<cache_dir>/huggingface`` (the reference's location) or, when that has
# no copy of the repository, $HF_HUB_CACHE / $HF_HOME/hub / ~/.cache/huggingface/hub.

HF_FORMATS = {"jsonl": (".jsonl", ".json"), "text": (".txt",), "parquet": (".parquet",), "csv": (".csv",)}


def hf_defaults(spec: dict) -> dict:
    """The HuggingFaceDatasetConfig keys with the reference's defaults filled in
    (train_files ["train.jsonl"] unless auto-discovered, text_fields ["text"], separator
    "\\n\\n", jsonl format); ``type = "nemotron_climb_mix"`` is the reference's preset
    (the ClimbMix parquet shards with pre-tokenised ``input_ids``)."""
    s = dict(spec)
    if s.get("type") == "nemotron_climb_mix":
        s = {"repo_id": "nvidia/Nemotron-CC/data/climb_mix", "format": "parquet", "train_files": [],
             "auto_discover_train_files": True, "text_fields": [], "sequence_field": "input_ids",
             "field_separator": " ", "revision": spec.get("revision"), "max_records": spec.get("max_records")}
    if "repo_id" not in s:
        raise ValueError("a huggingface dataset needs repo_id")
    s.setdefault("revision", None)
    s.setdefault("format", "jsonl")
    if s["format"] not in HF_FORMATS:
        raise ValueError(f"huggingface format must be one of {sorted(HF_FORMATS)}")
    s.setdefault("auto_discover_train_files", False)
    s.setdefault("train_files", [] if s["auto_discover_train_files"] else ["train.jsonl"])
    s.setdefault("validation_files", [])
    s.setdefault("text_fields", ["text"])
    s.setdefault("sequence_field", None)
    s.setdefault("field_separator", "\n\n")
    s.setdefault("template", None)
    s.setdefault("max_records", None)
    return s


def hf_snapshot_root(repo_id: str, revision: str | None, cache_dir: str | None = None) -> str:
    """The cached snapshot directory of a dataset repository: refs/<revision or main>
    names the snapshot; without that ref (or with a revision that is itself a snapshot
    id) the named or else the newest snapshot directory."""
    name = "datasets--" + repo_id.replace("/", "--")
    roots = []
    if cache_dir:
        roots.append(os.path.join(cache_dir, "huggingface"))
    env = os.environ.get("HF_HUB_CACHE") or (os.path.join(os.environ["HF_HOME"], "hub") if "HF_HOME" in os.environ
                                              else os.path.expanduser("~/.cache/huggingface/hub"))
    roots.append(env)
    for root in roots:
        repo = os.path.join(root, name)
        snaps = os.path.join(repo, "snapshots")
        if not os.path.isdir(snaps):
            continue
        ref = os.path.join(repo, "refs", revision or "main")
        if os.path.isfile(ref):
            sid = open(ref).read().strip()
            if os.path.isdir(os.path.join(snaps, sid)):
                return os.path.join(snaps, sid)
        if revision and os.path.isdir(os.path.join(snaps, revision)):
            return os.path.join(snaps, revision)
        ids = sorted(d for d in os.listdir(snaps) if os.path.isdir(os.path.join(snaps, d)))
        if ids:
            return os.path.join(snaps, ids[-1])
    raise FileNotFoundError(f"no cached snapshot of dataset {repo_id} under {roots} (no network: fill the "
                            "hub cache beforehand)")


def hf_files(spec: dict, root: str, split: str = "train") -> list[str]:
    """Files of the split, relative to the snapshot: the explicit list, else (train split,
    auto-discovery) every file of the format, restricted to paths naming "train" or
    "/default/" when any does (huggingface.rs resolve_hf_files)."""
    explicit = spec["train_files"] if split == "train" else spec["validation_files"]
    if explicit:
        return list(explicit)
    if split != "train" or not spec["auto_discover_train_files"]:
        return []
    ext = HF_FORMATS[spec["format"]]
    files = []
    for d, _, names in os.walk(root):
        for n in names:
            if n.endswith(ext):
                files.append(os.path.relpath(os.path.join(d, n), root).replace(os.sep, "/"))
    if any("train" in f or "/default/" in f for f in files):
        files = [f for f in files if "train" in f or "/default/" in f]
    if not files:
        raise FileNotFoundError(f"no {spec['format']} files discovered for dataset {spec['repo_id']}")
    return sorted(files)


def render_record(spec: dict, rec: dict) -> str | None:
    """A record's text: the template with {field} placeholders, else its text fields in
    order joined by the separator (records missing a field are skipped)."""
    tpl = spec.get("template")
    if tpl:
        out, i = [], 0
        while i < len(tpl):
            c = tpl[i]
            if c == "{":
                j = tpl.find("}", i)
                if j < 0:
                    raise ValueError("unclosed template placeholder")
                key = tpl[i + 1:j]
                if not key:
                    raise ValueError("empty template placeholder {}")
                if key not in rec:
                    return None
                out.append(str(rec[key]))
                i = j + 1
            else:
                out.append(c)
                i += 1
        return "".join(out)
    vals = []
    for f in spec["text_fields"]:
        if f not in rec or rec[f] is None:
            return None
        vals.append(str(rec[f]))
    return spec["field_separator"].join(vals)


def _hf_records(spec: dict, path: str):
    fmt = spec["format"]
    if fmt == "jsonl":
        with open(path, encoding="utf-8") as fh:
            for line in fh:
                line = line.strip()
                if line:
                    yield json.loads(line)
    elif fmt == "parquet":
        import pyarrow.parquet as pq

        for batch in pq.ParquetFile(path).iter_batches():
            yield from batch.to_pylist()
    elif fmt == "csv":
        import csv

        with open(path, encoding="utf-8", newline="") as fh:
            yield from csv.DictReader(fh)
    else:
        with open(path, encoding="utf-8", errors="replace") as fh:
            for line in fh:
                yield {"text": line.rstrip("\n")}


def prepare_hf_dataset(spec: dict, cache_dir: str, tokenizer: str | None = None, split: str = "train") -> str:
    """Render (or, with ``sequence_field``, take the pre-tokenised ids of) the split's
    records into a prepared token file like ``prepare_corpus``; returns its path."""
    spec = hf_defaults(spec)
    root = hf_snapshot_root(spec["repo_id"], spec["revision"], cache_dir)
    rel = hf_files(spec, root, split)
    if not rel:
        raise FileNotFoundError(f"dataset {spec['repo_id']}: no {split} files configured")
    files = [os.path.join(root, f) for f in rel]
    for f in files:
        if not os.path.exists(f):
            raise FileNotFoundError(f"{f} is not in the hub cache")
    sig = [[f, os.path.getsize(f), int(os.path.getmtime(f))] for f in files]
    tok = None
    if tokenizer and not spec["sequence_field"]:
        from ..utils.tokenizer import load_tokenizer

        tok = load_tokenizer(tokenizer)
        if tok.vocab_size > 65536:
            raise ValueError("token files hold uint16 ids: vocabulary must be <= 65536")
        sig.append([tokenizer, os.path.getsize(tokenizer), int(os.path.getmtime(tokenizer))])
    keyspec = {k: spec[k] for k in ("repo_id", "format", "text_fields", "sequence_field", "field_separator",
                                     "template", "max_records")}
    key = hashlib.sha256(json.dumps([sig, keyspec, split]).encode()).hexdigest()[:16]
    os.makedirs(cache_dir, exist_ok=True)
    out = os.path.join(cache_dir, f"hf-{key}.bin")
    man = out[:-4] + ".json"
    if os.path.exists(out) and os.path.exists(man):
        return out
    seq = spec["sequence_field"]
    sep = spec["field_separator"]
    width = 1 if (tok is None and not seq) else 2
    tmp = out + ".tmp"
    n = 0
    with open(tmp, "wb") as fh:
        for f in files:
            for rec in _hf_records(spec, f):
                if spec["max_records"] is not None and n >= spec["max_records"]:
                    break
                if seq:
                    ids = rec.get(seq)
                    if ids is None:
                        continue
                    a = np.asarray(ids, dtype=np.int64)
                    if a.size and (a.min() < 0 or a.max() > 65535):
                        raise ValueError(f"{seq}: token ids outside uint16")
                    fh.write(a.astype("<u2").tobytes())
                else:
                    text = render_record(spec, rec)
                    if text is None:
                        continue
                    if tok is None:
                        fh.write((sep if n else "").encode("utf-8") + text.encode("utf-8"))
                    else:
                        ids = (tok.encode(sep) if n else []) + tok.encode(text)
                        fh.write(np.asarray(ids, dtype="<u2").tobytes())
                n += 1
    os.replace(tmp, out)
    with open(man, "w") as fh:
        json.dump({"sources": sig, "repo_id": spec["repo_id"], "records": n, "split": split,
                   "bytes": os.path.getsize(out), "token_bytes": width,
                   "vocab": "bytes" if width == 1 else ("pretokenised" if seq else tok.vocab_size)}, fh, indent=2)
    return out
