"""Checkpoints and run directories.

Run layout (burn_dragon_language/src/checkpoint.rs:27-85,712-735; run_dirs.rs:37-46):

    <root>/<backend>/<run-name>/
        config.json                     model / optimizer / parallel / kernel spec
        training_config.json            the resolved training configuration
        tokenizer.json                  byte tokenizer description
        random_scaffold_manifest.json   (random-scaffold runs only)
        checkpoint/model-<step>.bpk     parameters
        checkpoint/optim-<step>.bpk     optimizer moments + step
        checkpoint/scheduler-<step>.bin learning-rate schedule position (JSON)
        checkpoint/runtime-state-<step>.bpk  streaming rho state, position, ...
        latest                          name of the newest checkpoint step

The root comes from ``BURN_DRAGON_RUN_ROOT`` (default ``runs``); ``BURN_DRAGON_RUN_DIR``
overrides the whole path and ``BURN_DRAGON_RUN_NAME`` the run name.

Tensor records are burnpack files (``train/burnpack.py``: the reference's container,
magic 0x4255524E, CBOR metadata, 256-byte aligned payloads), so a model record loads in
the reference's burnpack loaders and the reverse. The reference's own training
checkpoints are Burn ``BinFileRecorder`` records (``.bin``); those are not read here.
Records written by earlier versions of this package (``.bin`` in the safetensors
container: 8-byte little-endian header length, a JSON header, raw data) still load:
``load_tensors`` tells the two apart by the burnpack magic. Record names mirror the
reference's Burn record paths (``encoder``, ``embed.weight``, ``norm.gamma``, ...). Large
files split into burnpack parts with a SHA-256 manifest (burn_dragon_checkpoint/src/
parts.rs) and export at f16 (precision.rs). Retention keeps the newest two checkpoints
plus the best-validation one (schedule.rs:25,848-900).
"""

from __future__ import annotations

import json
import os
import re
import shutil
import struct
import threading
from dataclasses import asdict, is_dataclass

import torch

from . import burnpack as BP

SCHEMA_VERSION = 4  # burn_dragon_core/src/lib.rs:7
RECORD_EXT = ".bpk"

_DT = {
    torch.float32: "F32", torch.float16: "F16", torch.bfloat16: "BF16", torch.int64: "I64",
    torch.int32: "I32", torch.uint8: "U8", torch.float64: "F64", torch.bool: "BOOL",
}
_DT_INV = {v: k for k, v in _DT.items()}


# ------------------------------------------------------------------ tensor files
def save_tensors(path: str, tensors: dict[str, torch.Tensor], metadata: dict | None = None) -> None:
    """A ``.bpk`` path gets a burnpack file (metadata values JSON-encoded as text), any
    other path the safetensors container."""
    if path.endswith(".bpk"):
        BP.save_burnpack(path, tensors, {k: json.dumps(v) for k, v in (metadata or {}).items()})
        return
    header: dict = {}
    blobs = []
    off = 0
    for name in sorted(tensors):
        t = tensors[name].detach().contiguous().cpu()
        raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": _DT[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        header["__metadata__"] = {k: json.dumps(v) for k, v in metadata.items()}
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
    os.replace(tmp, path)


def _is_burnpack(path: str) -> bool:
    with open(path, "rb") as f:
        head = f.read(4)
    return len(head) == 4 and struct.unpack("<I", head)[0] == BP.MAGIC


def _meta_value(v: str):
    try:
        return json.loads(v)
    except (TypeError, ValueError):
        return v


def load_tensors(path: str, device=None) -> tuple[dict[str, torch.Tensor], dict]:
    """Tensors and metadata of a burnpack or safetensors record (told apart by the magic)."""
    if _is_burnpack(path):
        t, meta = BP.load_burnpack(path, device)
        return t, {k: _meta_value(v) for k, v in meta.items()}
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        data = f.read()
    meta = {k: json.loads(v) for k, v in header.pop("__metadata__", {}).items()}
    out = {}
    for name, info in header.items():
        a, b = info["data_offsets"]
        dt = _DT_INV[info["dtype"]]
        buf = bytearray(data[a:b])
        t = torch.frombuffer(buf, dtype=torch.uint8) if b > a else torch.empty(0, dtype=torch.uint8)
        t = t.view(dt).reshape(info["shape"]) if b > a else torch.empty(info["shape"], dtype=dt)
        out[name] = t.to(device) if device is not None else t
    return out, meta


def convert_precision(tensors: dict[str, torch.Tensor], dtype: torch.dtype) -> dict[str, torch.Tensor]:
    """Float tensors to `dtype` (f16 / bf16 export); integers are kept."""
    return {k: (v.to(dtype) if v.is_floating_point() else v) for k, v in tensors.items()}


def export_burnpack(model, path: str, f16: bool = False, part_mib: int | None = None,
                    metadata: dict | None = None) -> str:
    """Write the model's parameters under their record names as a burnpack deployment file
    (``<stem>.bpk``, or ``<stem>_f16.bpk`` with ``f16``), optionally split into parts of
    ``part_mib`` MiB with a ``.parts.json`` manifest. Returns the file path."""
    from ..models.bdh import record_name

    out = BP.precision_path(path, f16)
    tensors = {record_name(n): t.detach() for n, t in model.store.views(model.store.data).items()}
    if f16:
        tensors = {k: v.half() for k, v in tensors.items()}
    meta = {"schema_version": str(SCHEMA_VERSION), "producer": "burn_dragon_b200"}
    if f16:
        meta["precision"] = "f16"
    meta.update({k: str(v) for k, v in (metadata or {}).items()})
    BP.save_burnpack(out, tensors, meta)
    if part_mib:
        BP.write_parts(out, part_mib)
    return out


def load_model_burnpack(model, path: str, prefer_f16: bool = False) -> str:
    """Load a burnpack deployment file (or its parts manifest, or the preferred precision
    variant that exists) into the model's parameters; returns the file that was read."""
    from ..models.bdh import record_name

    cands = [path] if path.endswith(".parts.json") else BP.candidate_paths(path, prefer_f16)
    for c in cands:
        man = c if c.endswith(".parts.json") else BP.parts_manifest_path(c)
        if os.path.isfile(c) or os.path.isfile(man):
            tensors = BP.load_parts(man)[0] if os.path.isfile(man) and not os.path.isfile(c) else \
                (BP.load_parts(man)[0] if c.endswith(".parts.json") else BP.load_burnpack(c)[0])
            views = model.store.views(model.store.data)
            with torch.no_grad():
                for n, v in views.items():
                    src = tensors[record_name(n)]
                    if tuple(src.shape) != tuple(v.shape):
                        raise ValueError(f"{record_name(n)}: shape {tuple(src.shape)} != {tuple(v.shape)}")
                    v.copy_(src.to(v.device, v.dtype))
            model.store.refresh_shadow()
            return c
    raise FileNotFoundError(f"no burnpack at {path} (tried {cands})")


def save_parts(path: str, tensors: dict[str, torch.Tensor], max_part_bytes: int, metadata=None) -> dict:
    """A ``.bpk`` path: one burnpack file split into burnpack parts of at most
    ``max_part_bytes`` (rounded up to whole MiB) with the SHA-256 manifest
    ``<path>.parts.json``. Any other path: safetensors parts ``<path>.part-<i>`` with a
    name list in ``<path>.parts.json`` (the earlier container)."""
    if path.endswith(".bpk"):
        save_tensors(path, tensors, metadata)
        return BP.write_parts(path, max(1, -(-max_part_bytes // (1 << 20))))
    parts: list[list[str]] = [[]]
    size = 0
    for name in sorted(tensors):
        nb = tensors[name].numel() * tensors[name].element_size()
        if parts[-1] and size + nb > max_part_bytes:
            parts.append([])
            size = 0
        parts[-1].append(name)
        size += nb
    manifest = {"schema_version": SCHEMA_VERSION, "parts": []}
    for i, names in enumerate(parts):
        fname = f"{os.path.basename(path)}.part-{i:04d}"
        save_tensors(os.path.join(os.path.dirname(path), fname), {n: tensors[n] for n in names}, metadata)
        manifest["parts"].append({"file": fname, "tensors": names})
    with open(path + ".parts.json", "w") as f:
        json.dump(manifest, f, indent=2)
    return manifest


def load_parts(path: str, device=None) -> dict[str, torch.Tensor]:
    if path.endswith(".bpk"):
        return BP.load_parts(BP.parts_manifest_path(path), device)[0]
    with open(path + ".parts.json") as f:
        manifest = json.load(f)
    out: dict[str, torch.Tensor] = {}
    for part in manifest["parts"]:
        t, _ = load_tensors(os.path.join(os.path.dirname(path), part["file"]), device)
        out.update(t)
    return out


# ------------------------------------------------------------------ run directories
def _rel(p) -> str | None:
    """A relative path with empty, '.' and '..' parts dropped, or None if nothing is left."""
    if not p:
        return None
    parts = [x for x in str(p).replace("\\", "/").split("/") if x not in ("", ".", "..")]
    return os.path.join(*parts) if parts else None


def category_from_config_path(domain: str, path: str) -> str | None:
    """``.../config/<domain>/a/b/name.toml`` -> ``a/b/name``; ``.../config/local/[<domain>/]a/
    name.toml`` -> ``local/a/name`` (run_dirs.rs:83-141)."""
    comps = [c for c in os.path.normpath(path).split(os.sep) if c]
    stem = os.path.splitext(comps[-1])[0] if comps else None
    cfg_root = local_root = None
    for i in range(len(comps) - 1):
        if comps[i] == "config" and comps[i + 1] == domain:
            cfg_root = i
        if comps[i] == "config" and comps[i + 1] == "local":
            local_root = i
    if stem is None:
        return None
    if cfg_root is not None:
        return _rel("/".join(comps[cfg_root + 2:-1] + [stem]))
    if local_root is None:
        return None
    rest = comps[local_root + 2:-1]
    if rest and rest[0] == domain:
        rest = rest[1:]
    return _rel("/".join(["local"] + rest + [stem]))


def run_root_for(layout=None, config_paths=(), domain: str = "language", base: str | None = None) -> str:
    """``<base>/<domain>/[<category>]/[bundles/<b>]/[stages/<s>]/[variants/<v>]``; the
    category is ``layout.category`` or, with ``mirror_config_path``, derived from the last
    config path that sits under ``config/<domain>`` or ``config/local`` (run_dirs.rs:46-81)."""
    base = (layout.base_dir if layout is not None and layout.base_dir else None) or base or "runs"
    root = os.path.join(base, domain)
    if layout is None:
        return root
    cat = _rel(layout.category)
    if cat is None and layout.mirror_config_path:
        cat = next((c for c in (category_from_config_path(domain, p) for p in reversed(list(config_paths))) if c),
                   None)
    for prefix, part in (("", cat), ("bundles", _rel(layout.bundle)), ("stages", _rel(layout.stage)),
                         ("variants", _rel(layout.variant))):
        if part:
            root = os.path.join(root, prefix, part) if prefix else os.path.join(root, part)
    return root


def resolve_run_dir(backend: str = "cuda", run_name: str | None = None, root: str | None = None,
                    layout=None, config_paths=()) -> str:
    """``BURN_DRAGON_RUN_DIR`` if set; else ``<run root>/<backend>/<name>`` where the run
    root follows ``layout`` (base directory: ``layout.base_dir``, else ``root``, else
    ``BURN_DRAGON_RUN_ROOT``, else ``runs``). With a layout, the run root's ``latest`` file
    names the newest run (run_dirs.rs:196-212)."""
    if os.environ.get("BURN_DRAGON_RUN_DIR"):
        return os.environ["BURN_DRAGON_RUN_DIR"]
    base = root or os.environ.get("BURN_DRAGON_RUN_ROOT", "runs")
    name = run_name or os.environ.get("BURN_DRAGON_RUN_NAME") or "run"
    if layout is None:
        return os.path.join(base, backend, name)
    run_root = os.path.join(run_root_for(layout, config_paths, base=base), backend)
    return os.path.join(run_root, name)


def latest_run_dir(run_root: str) -> str | None:
    """The run named by ``<run_root>/latest``, if that directory exists."""
    p = os.path.join(run_root, "latest")
    if not os.path.isfile(p):
        return None
    name = open(p).read().strip()
    d = os.path.join(run_root, name)
    return d if name and os.path.isdir(d) else None


def write_latest_run(run_dir: str) -> None:
    """Record ``run_dir``'s name in its run root's ``latest`` file."""
    root = os.path.dirname(os.path.abspath(run_dir))
    os.makedirs(root, exist_ok=True)
    with open(os.path.join(root, "latest"), "w") as f:
        f.write(os.path.basename(os.path.abspath(run_dir)))


def _jsonable(x):
    if is_dataclass(x):
        return {k: _jsonable(v) for k, v in asdict(x).items()}
    if isinstance(x, dict):
        return {k: _jsonable(v) for k, v in x.items()}
    if isinstance(x, (list, tuple)):
        return [_jsonable(v) for v in x]
    return x


def _host_copy(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to("cpu", copy=True)


class RunDir:
    """``async_write``: ``save`` copies the tensors to host memory on the calling thread
    (the device work is ordered and finished before it returns) and writes the files on a
    background thread, so training continues during the disk writes; the next ``save``,
    ``load`` or ``wait`` waits for the previous write. The ``latest`` marker is written
    after the files it names (``[parallel.checkpoint] async_write``,
    burn_dragon_train/src/config/core.rs:217-222)."""

    def __init__(self, path: str, async_write: bool = False):
        self.path = path
        self.ckpt = os.path.join(path, "checkpoint")
        os.makedirs(self.ckpt, exist_ok=True)
        self.async_write = async_write
        self._writer: threading.Thread | None = None
        self._write_error: BaseException | None = None

    def wait(self) -> None:
        """Block until a background checkpoint write has finished; re-raise its error."""
        if self._writer is not None:
            self._writer.join()
            self._writer = None
        if self._write_error is not None:
            e, self._write_error = self._write_error, None
            raise RuntimeError("background checkpoint write failed") from e

    def write_json(self, name: str, obj) -> None:
        with open(os.path.join(self.path, name), "w") as f:
            json.dump(_jsonable(obj), f, indent=2, sort_keys=True)

    def read_json(self, name: str):
        with open(os.path.join(self.path, name)) as f:
            return json.load(f)

    def write_run_config(self, train_cfg) -> None:
        """config.json (RunConfigOutput-like spec) and training_config.json."""
        self.write_json("config.json", {
            "schema_version": SCHEMA_VERSION,
            "model_spec": train_cfg.model,
            "optimizer_spec": train_cfg.optimizer,
            "parallel_spec": train_cfg.parallel,
            "kernel_spec": {"backend": "sm_100a tcgen05", "dtype": "bf16 operands, fp32 accumulate/master"},
            "state_layout": {"rho": "[B, H, Nh, D] fp32 per layer"},
        })
        self.write_json("training_config.json", train_cfg)
        tok = getattr(train_cfg.dataset, "tokenizer", None)
        if tok:
            with open(tok) as f:
                self.write_json("tokenizer.json", json.load(f))
        else:
            self.write_json("tokenizer.json", {"type": "byte", "vocab_size": train_cfg.model.vocab_size})

    # ---- checkpoints
    def _p(self, kind: str, step: int, write: bool = False) -> str:
        """Record path: ``.bpk`` (burnpack); for reading, an earlier ``.bin`` record when
        no ``.bpk`` exists. The scheduler record is JSON in ``.bin``."""
        if kind == "scheduler":
            return os.path.join(self.ckpt, f"{kind}-{step}.bin")
        new = os.path.join(self.ckpt, f"{kind}-{step}{RECORD_EXT}")
        if write or os.path.exists(new):
            return new
        old = os.path.join(self.ckpt, f"{kind}-{step}.bin")
        return old if os.path.exists(old) else new

    def save(self, step: int, model, optimizer=None, scheduler: dict | None = None, runtime: dict | None = None,
             keep_last: int = 2, best_step: int | None = None, extra: dict | None = None, teacher=None,
             sharded: bool = False) -> None:
        """``extra``: further named tensors (the optional modules of ``DragonRuntime`` and
        their optimizer moments), stored as ``extra-<step>.bpk``. ``sharded``: the model
        and optimizer records were written per rank by ``save_shard``; write the rest."""
        from ..models.bdh import record_name

        self.wait()
        snap = _host_copy if self.async_write else (lambda t: t.detach())
        params = {} if sharded else {record_name(n): snap(t) for n, t in model.store.views(model.store.data).items()}
        optim = None
        if optimizer is not None and not sharded:
            optim = ({"m": snap(optimizer.m), "v": snap(optimizer.v)}, {"t": optimizer.t, "lr": optimizer.lr})
        rt = meta = None
        if runtime is not None:
            meta = {k: v for k, v in runtime.items() if k not in ("rhos", "state_tensors")}
            rt = {f"rho.{i}": snap(r) for i, r in enumerate(runtime.get("rhos") or [])}
            # the layer-loop variants' auxiliary memories, ``state.<layer>.<field>[.<key>]``
            rt.update({f"state.{k}": snap(v) for k, v in (runtime.get("state_tensors") or {}).items()})
        extra = {k: snap(v) for k, v in extra.items()} if extra else None
        # an EMA teacher (self-distillation, dynamics anchor, latent targets) is part of the
        # run's state: ``teacher-model-<step>.bin`` (burn_dragon_language/src/train/
        # runtime_checkpoint.rs:13-14)
        teach = {k: snap(v) for k, v in teacher.state_dict().items()} if teacher is not None else None
        scheduler = dict(scheduler or {})

        def write():
            if not sharded:
                save_tensors(self._p("model", step, True), params, {"schema_version": SCHEMA_VERSION, "step": step})
            if optim is not None and not sharded:
                save_tensors(self._p("optim", step, True), *optim)
            with open(self._p("scheduler", step), "w") as f:
                json.dump(scheduler, f)
            if rt is not None:
                save_tensors(self._p("runtime-state", step, True), rt, meta)
            if extra:
                save_tensors(self._p("extra", step, True), extra, {"schema_version": SCHEMA_VERSION})
            if teach:
                save_tensors(self._p("teacher-model", step, True), teach, {"schema_version": SCHEMA_VERSION})
            with open(os.path.join(self.path, "latest"), "w") as f:
                f.write(str(step))
            self._retain(keep_last, best_step)

        if not self.async_write:
            write()
            return

        def run():
            try:
                write()
            except BaseException as e:  # surfaced by the next wait()
                self._write_error = e

        self._writer = threading.Thread(target=run, name=f"checkpoint-{step}", daemon=False)
        self._writer.start()

    # ---- sharded records (``[parallel.checkpoint] format = "sharded_v2"``)
    def save_shard(self, step: int, rank: int, world: int, slices: list[tuple[int, int]], master: torch.Tensor,
                   m: torch.Tensor, v: torch.Tensor, numel: int, t: int) -> None:
        """One data-parallel rank's record of its own slices of the flat store: the fp32
        master and both AdamW moments (``model-<step>.shard-<r>-of-<W>.bpk``). Every rank
        writes its own file, in parallel, without gathering anything; ``load`` assembles
        them for any world size."""
        self.wait()
        vals = master.detach().reshape(-1)
        take = torch.cat([vals[a:b] for a, b in slices]) if slices else vals[:0]
        meta = {"schema_version": SCHEMA_VERSION, "step": step, "rank": rank, "world": world, "numel": numel,
                "t": t, "slices": [[int(a), int(b)] for a, b in slices]}
        save_tensors(os.path.join(self.ckpt, f"model-{step}.shard-{rank}-of-{world}{RECORD_EXT}"),
                     {"master": take, "m": m.detach().reshape(-1)[:take.numel()],
                      "v": v.detach().reshape(-1)[:take.numel()]}, meta)

    def shard_files(self, step: int) -> list[str]:
        pat = re.compile(rf"model-{step}\.shard-(\d+)-of-(\d+)\.bpk")
        return sorted((os.path.join(self.ckpt, fn) for fn in os.listdir(self.ckpt) if pat.fullmatch(fn)))

    def load_shards(self, step: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, int] | None:
        """(master, m, v, optimizer step) assembled from every shard file of ``step``, or
        None when the step has none. Checks that the shards cover the store exactly."""
        files = self.shard_files(step)
        if not files:
            return None
        full = mm = vv = None
        covered = 0
        t = 0
        worlds = set()
        for f in files:
            ten, meta = load_tensors(f)
            worlds.add(int(meta["world"]))
            n = int(meta["numel"])
            if full is None:
                full, mm, vv = torch.zeros(n), torch.zeros(n), torch.zeros(n)
            off = 0
            for a, b in meta["slices"]:
                k = b - a
                full[a:b] = ten["master"][off:off + k]
                mm[a:b] = ten["m"][off:off + k]
                vv[a:b] = ten["v"][off:off + k]
                off += k
                covered += k
            t = int(meta["t"])
        if len(worlds) != 1 or len(files) != next(iter(worlds)):
            raise ValueError(f"checkpoint step {step}: incomplete shard set {files}")
        if covered != full.numel():
            raise ValueError(f"checkpoint step {step}: shards cover {covered} of {full.numel()} elements")
        return full, mm, vv, t

    def steps(self) -> list[int]:
        out = []
        for fn in os.listdir(self.ckpt):
            m = re.fullmatch(r"model-(\d+)(?:\.shard-0-of-\d+)?\.(?:bin|bpk)", fn)
            if m:
                out.append(int(m.group(1)))
        return sorted(set(out))

    def latest(self) -> int | None:
        p = os.path.join(self.path, "latest")
        if os.path.exists(p):
            return int(open(p).read().strip())
        s = self.steps()
        return s[-1] if s else None

    def _retain(self, keep_last: int, best_step: int | None) -> None:
        steps = self.steps()
        keep = set(steps[-keep_last:]) | ({best_step} if best_step is not None else set())
        for s in steps:
            if s in keep:
                continue
            for kind in ("model", "optim", "scheduler", "runtime-state", "extra", "teacher-model"):
                for ext in (".bin", RECORD_EXT):
                    p = os.path.join(self.ckpt, f"{kind}-{s}{ext}")
                    if os.path.exists(p):
                        os.remove(p)
            for p in self.shard_files(s):
                os.remove(p)

    def load_teacher(self, step: int, teacher) -> bool:
        """Restore an EMA teacher saved with ``save(..., teacher=)``; False if absent."""
        self.wait()
        p = self._p("teacher-model", step)
        if not os.path.exists(p):
            return False
        sd, _ = load_tensors(p)
        teacher.load_state_dict({k: v.to(t.device, t.dtype) for (k, v), t in
                                 zip(sd.items(), [teacher.state_dict()[k] for k in sd])}, strict=False)
        return True

    def load(self, step: int | None, model, optimizer=None, device=None) -> dict:
        """Restore model (and optimizer) state; returns {'scheduler', 'runtime'}."""
        from ..models.bdh import record_name

        self.wait()
        step = self.latest() if step is None else step
        if step is None:
            raise FileNotFoundError(f"no checkpoint in {self.ckpt}")
        shards = None if os.path.exists(self._p("model", step)) else self.load_shards(step)
        if shards is not None:
            full, mm, vv, t = shards
            n = model.store.numel
            if full.numel() < n:
                raise ValueError(f"sharded checkpoint holds {full.numel()} elements, the model {n}")
            with torch.no_grad():
                model.store.data[:n].copy_(full[:n].to(model.store.data.device))
            model.store.refresh_shadow()
            if optimizer is not None:
                optimizer.m[:n].copy_(mm[:n].to(optimizer.m.device))
                optimizer.v[:n].copy_(vv[:n].to(optimizer.v.device))
                optimizer.t = t
        else:
            tensors, meta = load_tensors(self._p("model", step))
            if int(meta.get("schema_version", SCHEMA_VERSION)) != SCHEMA_VERSION:
                raise ValueError("checkpoint schema version mismatch")
            views = model.store.views(model.store.data)
            with torch.no_grad():
                for n, v in views.items():
                    src = tensors[record_name(n)]
                    if tuple(src.shape) != tuple(v.shape):
                        raise ValueError(f"{record_name(n)}: checkpoint shape {tuple(src.shape)} != {tuple(v.shape)}")
                    v.copy_(src.to(v.device, v.dtype))
            model.store.refresh_shadow()
        if shards is None and optimizer is not None and os.path.exists(self._p("optim", step)):
            o, ometa = load_tensors(self._p("optim", step))
            optimizer.m.copy_(o["m"].to(optimizer.m.device))
            optimizer.v.copy_(o["v"].to(optimizer.v.device))
            optimizer.t = int(ometa["t"])
        out = {"step": step, "scheduler": {}, "runtime": None, "extra": None}
        ep = self._p("extra", step)
        if os.path.exists(ep):
            out["extra"] = load_tensors(ep, device)[0]
        sp = self._p("scheduler", step)
        if os.path.exists(sp):
            out["scheduler"] = json.load(open(sp))
        rp = self._p("runtime-state", step)
        if os.path.exists(rp):
            rt, rmeta = load_tensors(rp, device)
            nrho = sum(1 for k in rt if k.startswith("rho."))
            rhos = [rt[f"rho.{i}"] for i in range(nrho)] or None
            runtime = dict(rmeta)
            runtime["rhos"] = rhos
            st = {k[len("state."):]: v for k, v in rt.items() if k.startswith("state.")}
            if st:
                runtime["state_tensors"] = st
            out["runtime"] = runtime
        return out

    def remove(self) -> None:
        shutil.rmtree(self.path, ignore_errors=True)
