"""Burnpack tensor files: the reference's deployment / checkpoint container.

File layout (all integers little-endian), as the reference writes and reads it
(burn_dragon_checkpoint/src/parts.rs:15-16,80-90,670-760):

    offset 0   u32  magic 0x4255524E
    offset 4   u16  format version
    offset 6   u32  metadata size S (bytes)
    offset 10  S bytes of CBOR: {"tensors": {name: {"dtype", "shape", "data_offsets"}},
                                 "metadata": {str: str}}
    then zero padding up to the data section, which starts at the next multiple of 256
    bytes; every tensor payload starts at a multiple of 256 within the data section and
    ``data_offsets`` = [start, end) relative to the data section.

``dtype`` is the name of Burn's ``DType`` variant as a CBOR text string ("F32", "F16",
"BF16", "I64", ...). The metadata map is free-form text; a precision conversion adds
``precision`` = "f16" / "f32" (precision.rs:56-133).

Parts (parts.rs:137-270,835-1025): ``<name>.parts.json`` next to the file lists
``<name>.part-00000.bpk``, ... Each part is itself a burnpack holding a run of the
source's tensors (in data-offset order) packed from offset 0; a part is closed before
the tensor that would push it past ``max_part_bytes`` (a tensor larger than the limit
gets a part of its own). The manifest records version 1, the source file name and its
modification time in ms, the source size, the part limit in bytes and, per part, its
file name, size, SHA-256 and tensor count. A reader checks every part's size and hash.

Precision variants (precision.rs:41-54, policy.rs:1-100): ``<stem>_f16.bpk`` next to
``<stem>.bpk``; float tensors converted, integer tensors kept.

CBOR (RFC 8949) is encoded and decoded here for the subset the format uses: unsigned /
negative integers, text and byte strings, arrays, maps, booleans, null and floats.
"""

from __future__ import annotations

import hashlib
import json
import os
import struct

import numpy as np
import torch

MAGIC = 0x4255524E
HEADER_SIZE = 10
ALIGN = 256
FORMAT_VERSION = 1
F16_SUFFIX = "_f16"

_DT = {torch.float32: "F32", torch.float16: "F16", torch.bfloat16: "BF16", torch.float64: "F64",
       torch.int64: "I64", torch.int32: "I32", torch.int16: "I16", torch.int8: "I8", torch.uint8: "U8",
       torch.bool: "Bool"}
_DT_INV = {v: k for k, v in _DT.items()}


# ------------------------------------------------------------------ CBOR subset
def _head(major: int, n: int) -> bytes:
    if n < 24:
        return bytes([(major << 5) | n])
    if n < 1 << 8:
        return bytes([(major << 5) | 24, n])
    if n < 1 << 16:
        return bytes([(major << 5) | 25]) + struct.pack(">H", n)
    if n < 1 << 32:
        return bytes([(major << 5) | 26]) + struct.pack(">I", n)
    return bytes([(major << 5) | 27]) + struct.pack(">Q", n)


def cbor_dumps(obj) -> bytes:
    """Definite-length CBOR of None / bool / int / float / str / bytes / list / tuple /
    dict (map keys in insertion order)."""
    if obj is None:
        return b"\xf6"
    if obj is True:
        return b"\xf5"
    if obj is False:
        return b"\xf4"
    if isinstance(obj, int):
        return _head(0, obj) if obj >= 0 else _head(1, -1 - obj)
    if isinstance(obj, float):
        return b"\xfb" + struct.pack(">d", obj)
    if isinstance(obj, str):
        raw = obj.encode()
        return _head(3, len(raw)) + raw
    if isinstance(obj, (bytes, bytearray)):
        return _head(2, len(obj)) + bytes(obj)
    if isinstance(obj, (list, tuple)):
        return _head(4, len(obj)) + b"".join(cbor_dumps(x) for x in obj)
    if isinstance(obj, dict):
        return _head(5, len(obj)) + b"".join(cbor_dumps(k) + cbor_dumps(v) for k, v in obj.items())
    raise TypeError(f"cannot CBOR-encode {type(obj).__name__}")


def cbor_loads(data: bytes):
    obj, pos = _decode(memoryview(data), 0)
    if pos != len(data):
        raise ValueError(f"trailing bytes after CBOR item ({len(data) - pos})")
    return obj


def _arg(buf, pos: int, info: int) -> tuple[int, int]:
    if info < 24:
        return info, pos
    if info == 24:
        return buf[pos], pos + 1
    if info == 25:
        return struct.unpack_from(">H", buf, pos)[0], pos + 2
    if info == 26:
        return struct.unpack_from(">I", buf, pos)[0], pos + 4
    if info == 27:
        return struct.unpack_from(">Q", buf, pos)[0], pos + 8
    raise ValueError(f"unsupported CBOR length encoding {info}")


def _decode(buf, pos: int):
    ib = buf[pos]
    pos += 1
    major, info = ib >> 5, ib & 31
    if major == 7:
        if info == 20:
            return False, pos
        if info == 21:
            return True, pos
        if info in (22, 23):
            return None, pos
        if info == 25:
            return float(np.frombuffer(bytes(buf[pos:pos + 2]), dtype=">f2")[0]), pos + 2
        if info == 26:
            return struct.unpack_from(">f", buf, pos)[0], pos + 4
        if info == 27:
            return struct.unpack_from(">d", buf, pos)[0], pos + 8
        raise ValueError(f"unsupported CBOR simple value {info}")
    if info == 31:
        raise ValueError("indefinite-length CBOR items are not used by burnpack")
    n, pos = _arg(buf, pos, info)
    if major == 0:
        return n, pos
    if major == 1:
        return -1 - n, pos
    if major == 2:
        return bytes(buf[pos:pos + n]), pos + n
    if major == 3:
        return bytes(buf[pos:pos + n]).decode(), pos + n
    if major == 4:
        out = []
        for _ in range(n):
            v, pos = _decode(buf, pos)
            out.append(v)
        return out, pos
    if major == 5:
        out = {}
        for _ in range(n):
            k, pos = _decode(buf, pos)
            v, pos = _decode(buf, pos)
            out[k] = v
        return out, pos
    if major == 6:  # tag: keep the tagged item
        return _decode(buf, pos)
    raise ValueError(f"unsupported CBOR major type {major}")


# ------------------------------------------------------------------ files
def _align(x: int, a: int = ALIGN) -> int:
    return -(-x // a) * a


def _raw(t: torch.Tensor) -> bytes:
    t = t.detach().contiguous().cpu()
    return t.view(torch.uint8).numpy().tobytes() if t.numel() else b""


def _write(path: str, version: int, descriptors: dict, meta: dict, payloads: list[bytes]) -> None:
    """Header, CBOR metadata, padding to the data section, then the payloads at their
    descriptors' offsets (descriptors in the payloads' order)."""
    md = cbor_dumps({"tensors": dict(sorted(descriptors.items())), "metadata": dict(sorted(meta.items()))})
    data_start = _align(HEADER_SIZE + len(md))
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<IHI", MAGIC, version, len(md)))
        f.write(md)
        f.write(b"\0" * (data_start - HEADER_SIZE - len(md)))
        written = 0
        for (name, d), raw in zip(descriptors.items(), payloads):
            a, b = d["data_offsets"]
            if b - a != len(raw):
                raise ValueError(f"tensor {name}: payload length {len(raw)} != {b - a}")
            f.write(b"\0" * (a - written))
            f.write(raw)
            written = b
    os.replace(tmp, path)


def save_burnpack(path: str, tensors: dict[str, torch.Tensor], metadata: dict | None = None,
                  version: int = FORMAT_VERSION) -> str:
    """Write ``tensors`` (name -> CPU or CUDA tensor) as one burnpack file. Payloads are
    laid out in name order, each at a 256-byte boundary; metadata values become text."""
    descriptors, payloads, off = {}, [], 0
    for name in sorted(tensors):
        t = tensors[name]
        raw = _raw(t)
        a = _align(off)
        descriptors[name] = {"dtype": _DT[t.dtype], "shape": [int(s) for s in t.shape], "data_offsets": [a, a + len(raw)]}
        payloads.append(raw)
        off = a + len(raw)
    meta = {str(k): (v if isinstance(v, str) else json.dumps(v)) for k, v in (metadata or {}).items()}
    _write(path, version, descriptors, meta, payloads)
    return path


def read_header(path: str) -> tuple[int, int, dict]:
    """(version, metadata size, decoded metadata) of a burnpack file."""
    with open(path, "rb") as f:
        head = f.read(HEADER_SIZE)
        if len(head) != HEADER_SIZE:
            raise ValueError(f"{path}: shorter than a burnpack header")
        magic, version, size = struct.unpack("<IHI", head)
        if magic != MAGIC:
            raise ValueError(f"{path}: invalid burnpack magic {magic:#x} (expected {MAGIC:#x})")
        md = cbor_loads(f.read(size))
    if not isinstance(md, dict) or "tensors" not in md:
        raise ValueError(f"{path}: burnpack metadata has no tensor table")
    md.setdefault("metadata", {})
    return version, size, md


def _dtype_of(v) -> torch.dtype:
    name = v if isinstance(v, str) else (next(iter(v)) if isinstance(v, dict) and v else str(v))
    if name not in _DT_INV:
        raise ValueError(f"unsupported burnpack dtype {v!r}")
    return _DT_INV[name]


def load_burnpack(path: str, device=None) -> tuple[dict[str, torch.Tensor], dict]:
    """(tensors, metadata) of a burnpack file."""
    version, size, md = read_header(path)
    data_start = _align(HEADER_SIZE + size)
    out = {}
    with open(path, "rb") as f:
        for name, d in md["tensors"].items():
            a, b = (int(x) for x in d["data_offsets"])
            dt = _dtype_of(d["dtype"])
            shape = [int(s) for s in d["shape"]]
            f.seek(data_start + a)
            buf = bytearray(f.read(b - a))
            if len(buf) != b - a:
                raise ValueError(f"{path}: tensor {name} is truncated")
            t = torch.frombuffer(buf, dtype=torch.uint8).view(dt).reshape(shape) if b > a else \
                torch.empty(shape, dtype=dt)
            out[name] = t.to(device) if device is not None else t
    return out, dict(md["metadata"])


# ------------------------------------------------------------------ parts
def parts_manifest_path(path: str) -> str:
    return os.path.join(os.path.dirname(path), os.path.basename(path) + ".parts.json")


def _sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def _part_size(records: list, meta: dict) -> int:
    tensors, off = {}, 0
    for name, d in records:
        n = d["data_offsets"][1] - d["data_offsets"][0]
        a = _align(off)
        tensors[name] = {**d, "data_offsets": [a, a + n]}
        off = a + n
    md = cbor_dumps({"tensors": dict(sorted(tensors.items())), "metadata": dict(sorted(meta.items()))})
    return _align(HEADER_SIZE + len(md)) + off


def write_parts(path: str, max_part_mib: int = 64) -> dict:
    """Split the burnpack ``path`` into parts of at most ``max_part_mib`` MiB each and write
    ``<path>.parts.json``; returns the manifest."""
    version, size, md = read_header(path)
    data_start = _align(HEADER_SIZE + size)
    meta = dict(md["metadata"])
    limit = max(1, int(max_part_mib)) * (1 << 20)
    records = sorted(md["tensors"].items(), key=lambda kv: kv[1]["data_offsets"][0])
    if not records:
        raise ValueError(f"{path}: no tensors to split")
    groups, cur = [], []
    for rec in records:
        if cur and _part_size(cur + [rec], meta) > limit:
            groups.append(cur)
            cur = [rec]
        else:
            cur = cur + [rec]
    groups.append(cur)
    base = os.path.basename(path)
    entries = []
    with open(path, "rb") as src:
        for i, group in enumerate(groups):
            part_name = f"{base}.part-{i:05d}.bpk"
            part_path = os.path.join(os.path.dirname(path), part_name)
            descriptors, payloads, off = {}, [], 0
            for name, d in group:
                a0, b0 = d["data_offsets"]
                src.seek(data_start + a0)
                raw = src.read(b0 - a0)
                a = _align(off)
                descriptors[name] = {**d, "data_offsets": [a, a + len(raw)]}
                payloads.append(raw)
                off = a + len(raw)
            _write(part_path, version, descriptors, meta, payloads)
            entries.append({"path": part_name, "bytes": os.path.getsize(part_path), "sha256": _sha256(part_path),
                            "tensors": len(group)})
    manifest = {"version": 1, "source_file": base,
                "source_modified_unix_ms": int(os.path.getmtime(path) * 1000),
                "total_bytes": os.path.getsize(path), "max_part_bytes": limit, "parts": entries}
    with open(parts_manifest_path(path), "w") as f:
        json.dump(manifest, f, indent=2)
    return manifest


def load_parts(manifest_path: str, device=None) -> tuple[dict[str, torch.Tensor], dict]:
    """Tensors and metadata from every part a manifest lists, after checking each part's
    size and SHA-256."""
    with open(manifest_path) as f:
        manifest = json.load(f)
    root = os.path.dirname(manifest_path)
    tensors, meta = {}, {}
    for e in manifest.get("parts", []):
        p = os.path.join(root, e["path"])
        if not os.path.isfile(p):
            raise FileNotFoundError(f"burnpack part missing: {p}")
        if e.get("bytes") and os.path.getsize(p) != int(e["bytes"]):
            raise ValueError(f"burnpack part {p}: size {os.path.getsize(p)} != {e['bytes']}")
        if e.get("sha256") and _sha256(p) != e["sha256"]:
            raise ValueError(f"burnpack part {p}: SHA-256 mismatch")
        t, m = load_burnpack(p, device)
        tensors.update(t)
        meta.update(m)
    return tensors, meta


# ------------------------------------------------------------------ precision variants
def precision_path(path: str, f16: bool) -> str:
    """``<stem>.bpk`` or ``<stem>_f16.bpk`` (the extension forced to .bpk)."""
    root, ext = os.path.splitext(path)
    if ext.lower() != ".bpk":
        root = path if ext == "" else root
    return root + (F16_SUFFIX if f16 else "") + ".bpk"


def convert_precision(src: str, out: str, precision: str) -> str:
    """Rewrite a burnpack with its float tensors in ``precision`` ("f16" or "f32");
    integer tensors are kept and the metadata records ``precision``."""
    if precision not in ("f16", "f32"):
        raise ValueError("precision must be 'f16' or 'f32'")
    target = torch.float16 if precision == "f16" else torch.float32
    version, _, _ = read_header(src)
    tensors, meta = load_burnpack(src)
    conv = {k: (v.to(target) if v.is_floating_point() else v) for k, v in tensors.items()}
    meta["precision"] = precision
    save_burnpack(out, conv, meta, version=version)
    return out


def candidate_paths(path: str, prefer_f16: bool = False) -> list[str]:
    """Load order of the precision variants of ``path``."""
    a, b = precision_path(path, False), precision_path(path, True)
    return [b, a] if prefer_f16 else [a, b]


# ------------------------------------------------------------------ bootstrap from a URL
# Resolve a model's weights from a local cache, fetching them from a remote base URL when
# the cache has neither a complete parts set nor a monolithic file (the reference's
# bootstrap, burn_dragon_checkpoint/src/bootstrap.rs:19-330): for each precision variant in
# the load order, a complete cached parts manifest wins, then a cached monolithic file,
# then the remote parts manifest (<url>.parts.json) with every part fetched and checked
# against its size / SHA-256, then the remote monolithic file. URLs are http(s):// or
# file:// (urllib); writes are atomic (temporary file + rename).

def default_cache_root() -> str:
    """$BURN_DRAGON_CACHE_DIR, else ~/.cache/burn_dragon/models."""
    env = os.environ.get("BURN_DRAGON_CACHE_DIR")
    if env:
        return env
    return os.path.join(os.path.expanduser("~"), ".cache", "burn_dragon", "models")


def _url_with_suffix(url: str, suffix: str) -> str:
    head, _, tail = url.rpartition("/")
    stem, dot, ext = tail.rpartition(".")
    if dot and not stem.endswith(suffix):
        tail = f"{stem}{suffix}.{ext}"
    elif not dot and not tail.endswith(suffix):
        tail = tail + suffix
    return f"{head}/{tail}" if head else tail


def candidate_urls(base_url: str, prefer_f16: bool = False) -> list[str]:
    """The remote burnpack URLs in load order (``.bpk`` appended when missing)."""
    f32 = base_url if base_url.endswith(".bpk") else base_url + ".bpk"
    f16 = _url_with_suffix(f32, F16_SUFFIX)
    if f16 == f32:
        return [f32]
    return [f16, f32] if prefer_f16 else [f32, f16]


def _entry_url(manifest_url: str, entry: str) -> str:
    if entry.startswith(("http://", "https://", "file://")):
        return entry
    base = manifest_url.rpartition("/")[0]
    return f"{base.rstrip('/')}/{entry.lstrip('/')}" if base else entry.lstrip("/")


def _fetch(url: str, timeout: float = 60.0) -> bytes | None:
    """The body at ``url``, or None when it does not exist (HTTP 404 / missing file)."""
    import urllib.error
    import urllib.request

    try:
        with urllib.request.urlopen(url, timeout=timeout) as r:
            return r.read()
    except urllib.error.HTTPError as e:
        if e.code == 404:
            return None
        raise
    except urllib.error.URLError as e:
        if isinstance(e.reason, FileNotFoundError) or "No such file" in str(e.reason):
            return None
        raise


def _write_atomic(path: str, data: bytes) -> None:
    os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
    tmp = f"{path}.tmp-{os.getpid()}"
    with open(tmp, "wb") as f:
        f.write(data)
    os.replace(tmp, path)


def _part_ok(path: str, entry: dict) -> bool:
    if not os.path.isfile(path):
        return False
    if entry.get("bytes") and os.path.getsize(path) != int(entry["bytes"]):
        return False
    return not entry.get("sha256") or _sha256(path) == entry["sha256"]


def manifest_complete(manifest_path: str) -> bool:
    """Every part the manifest lists is present with its size and checksum."""
    if not os.path.isfile(manifest_path):
        return False
    with open(manifest_path) as f:
        man = json.load(f)
    root = os.path.dirname(manifest_path)
    parts = man.get("parts", [])
    return bool(parts) and all(_part_ok(os.path.join(root, e["path"]), e) for e in parts)


def resolve_or_bootstrap(local_base: str, remote_base_url: str, cache_root: str | None = None,
                         prefer_parts: bool = True, verify_checksums: bool = True, prefer_f16: bool = False,
                         progress=None) -> str:
    """The local burnpack path to load (``load_parts`` on its ``.parts.json`` when that is
    complete, else ``load_burnpack``), fetched from ``remote_base_url`` when not cached. A
    relative ``local_base`` lives under ``cache_root`` (default ``default_cache_root()``)."""
    say = progress or (lambda msg: None)
    root = cache_root or default_cache_root()
    os.makedirs(root, exist_ok=True)
    base = local_base if os.path.isabs(local_base) else os.path.join(root, local_base)
    last = None
    for local, remote in zip(candidate_paths(base, prefer_f16), candidate_urls(remote_base_url, prefer_f16)):
        man_path = parts_manifest_path(local)
        if manifest_complete(man_path):
            say(f"using cached multipart burnpack {man_path}")
            return local
        if os.path.isfile(local):
            say(f"using cached monolithic burnpack {local}")
            return local
        if prefer_parts:
            murl = remote + ".parts.json"
            try:
                body = _fetch(murl)
            except OSError:
                body = None
            if body is not None:
                _write_atomic(man_path, body)
                man = json.loads(body)
                ok = bool(man.get("parts"))
                for i, e in enumerate(man.get("parts", [])):
                    p = os.path.join(os.path.dirname(man_path), e["path"])
                    if _part_ok(p, e):
                        continue
                    say(f"downloading burnpack part {i + 1}/{len(man['parts'])}")
                    try:
                        data = _fetch(_entry_url(murl, e["path"]))
                    except OSError:
                        data = None
                    if data is None:
                        ok = False
                        break
                    _write_atomic(p, data)
                    if verify_checksums and not _part_ok(p, e):
                        ok = False
                        break
                if ok and manifest_complete(man_path):
                    return local
        say(f"downloading monolithic burnpack {remote}")
        try:
            data = _fetch(remote)
        except OSError as e:
            last = str(e)
            continue
        if data is None:
            last = f"{remote}: not found"
            continue
        _write_atomic(local, data)
        return local
    raise FileNotFoundError(last or f"failed to resolve burnpack weights for {base}")


def load_resolved(path: str, device=None) -> tuple[dict[str, torch.Tensor], dict]:
    """Load what ``resolve_or_bootstrap`` returned: its complete parts set, else the file."""
    man = parts_manifest_path(path)
    if manifest_complete(man):
        return load_parts(man, device)
    return load_burnpack(path, device)
