"""Top-level training driver: ``train(TrainingConfig)``.

Mirrors the reference's ``train_backend`` flow (burn_dragon_language/src/train/
backend.rs:1187-1915): resolve the parallel runtime from WORLD_SIZE / RANK / LOCAL_RANK,
seed, create the run directory and write ``config.json`` / ``training_config.json`` /
``tokenizer.json`` (and ``random_scaffold_manifest.json``), build the model and AdamW,
resume from the newest checkpoint, then run the step loop with metrics, periodic
validation and checkpoints, the non-finite-loss interrupter and peer heartbeats.

Parallel modes (``[parallel] mode``): ``single``; ``ddp`` (NVLink peer-memory step on
CUDA, gloo/NCCL all-reduce otherwise); ``tensor_parallel_neuron`` (head-aligned neuron
sharding); ``pipeline`` (``[parallel.pipeline] schedule / micro_batches``); ``fsdp`` maps
to ``ddp`` with the partitioned (sharded-moment) optimizer step.

Sequence batching: ``random`` windows, or ``streaming`` with stateful TBPTT
(``tbptt_chunk_size``, ``tbptt_persist_across_steps``): every step trains the next chunk
of each stream with the linear-attention state carried (detached) from the previous
chunk, reset at stream starts (burn_dragon_language/src/train/steps.rs:2698-2731,
11860-11960); the state is saved in ``runtime-state-<step>.bpk``.
"""

from __future__ import annotations

import os
import time

import torch
import torch.distributed as dist

from ..config import TrainingConfig
from ..models.state import ModelState
from ..parallel.fault import Heartbeat, NonFiniteGuard, PeerFailure
from . import checkpoint as C
from .data import FileBytes, RandomBytes, StreamingBytes
from .metrics import MetricsLogger, StageProfiler, theoretical_forward_flops
from .trainer import Trainer, init_distributed


def _device(local: int, backend: str | None = None) -> torch.device:
    """``backend="cpu"`` keeps a run on the host even where a GPU is present."""
    if backend == "cpu":
        return torch.device("cpu")
    if backend == "cuda" and not torch.cuda.is_available():
        raise RuntimeError("backend cuda requested but no CUDA device is visible")
    return torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")


def train(cfg: TrainingConfig, run_name: str | None = None, resume: bool = True, backend: str | None = None) -> dict:
    rank, world, local = init_distributed()
    dev = _device(local, backend)
    if dev.type == "cuda":
        torch.cuda.set_device(dev)
    t = cfg.training
    mode = cfg.parallel.mode
    torch.manual_seed(t.seed + rank)
    ck = cfg.parallel.checkpoint or {}
    ck_format = ck.get("format", "unsharded_v1")
    if ck_format not in ("unsharded_v1", "sharded_v2"):
        raise ValueError(f"parallel.checkpoint.format {ck_format!r}: unsharded_v1 or sharded_v2")
    lm = t.launch_mode
    if lm in ("fresh", "init_from_checkpoint"):
        resume = False
    if lm == "resume_exact_run":
        if not os.path.isdir(t.resume_run_dir):
            raise ValueError(f"training.resume_run_dir does not exist or is not a directory: {t.resume_run_dir}")
        run_path = t.resume_run_dir
    else:
        if lm in ("fresh", "init_from_checkpoint") and not run_name and not os.environ.get("BURN_DRAGON_RUN_NAME"):
            # a fresh launch gets a run directory of its own (run_dirs.rs:143-160); rank 0
            # names it and the others take that name
            base = f"run-{time.strftime('%Y%m%d-%H%M%S')}-{os.getpid()}"
            name, i = [base], 1
            while os.path.exists(C.resolve_run_dir(dev.type, name[0], layout=cfg.run_layout,
                                                   config_paths=cfg.config_paths)):
                i += 1
                name = [f"{base}-{i}"]
            if world > 1:
                dist.broadcast_object_list(name, src=0)
            run_name = name[0]
        run_path = C.resolve_run_dir(dev.type, run_name, layout=cfg.run_layout, config_paths=cfg.config_paths)
        if lm == "resume_latest_checkpoint_if_present" and not run_name:
            prev = C.latest_run_dir(os.path.dirname(os.path.abspath(run_path)))
            if prev is not None and C.RunDir(prev).steps():
                run_path = prev
    run = C.RunDir(run_path, async_write=bool(ck.get("async_write", False)))
    if rank == 0 and not os.environ.get("BURN_DRAGON_RUN_DIR"):
        C.write_latest_run(run.path)
    if rank == 0:
        run.write_run_config(cfg)
        if cfg.model.random_scaffold.enabled:
            from ..models import scaffold as S

            man_path = os.path.join(run.path, "random_scaffold_manifest.json")
            if os.path.exists(man_path):
                import json

                S.check_manifest(json.load(open(man_path)), cfg.model)
            else:
                S.write_manifest(man_path, cfg.model)
    o = cfg.optimizer
    comm = None
    if mode in ("ddp", "fsdp") and world > 1 and dev.type == "cuda" and o.name != "eggroll":
        # the NVLink step implements global-norm clipping; element-wise value clipping of the
        # mean gradient runs on the NCCL path
        comm = "nvlink" if o.grad_clip_value is None else "nccl"
        # [parallel.data] transport = "nvls": the same step through NVLink multicast objects
        # (in-switch gradient sums; measured faster than peer loads at 8 ranks, slower at 2)
        if comm == "nvlink" and cfg.parallel.data.get("transport", "p2p") == "nvls":
            comm = "nvls"
    micro = int(cfg.parallel.tensor.get("micro_batches", t.gradient_accumulation_steps))
    tp_arg: bool | int = mode == "tensor_parallel_neuron"
    if mode == "hybrid_2d":
        tp_arg = int(cfg.parallel.tensor.get("size", 8))
        comm = "nvlink" if o.grad_clip_value is None and dev.type == "cuda" else None
    seq_par = bool(cfg.parallel.tensor.get("sequence_parallel", False))
    if seq_par and not tp_arg:
        raise ValueError("parallel.tensor.sequence_parallel needs a tensor-parallel mode "
                         "(tensor_parallel_neuron or hybrid_2d)")
    if cfg.dataset.type in ("huggingface", "nemotron_climb_mix"):
        from .datasets import prepare_hf_dataset

        if cfg.dataset.type == "huggingface":
            spec = dict(cfg.dataset.huggingface or {})
        else:
            spec = {"type": "nemotron_climb_mix", "revision": cfg.dataset.revision,
                    "max_records": cfg.dataset.max_records}
        splits = ["train"] + (["validation"] if spec.get("validation_files") and not cfg.dataset.validation else [])
        if rank == 0:
            for sp in splits:
                prepare_hf_dataset(spec, cfg.dataset.cache_dir, tokenizer=cfg.dataset.tokenizer, split=sp)
        if world > 1 and dist.is_initialized():
            dist.barrier()
        prepared, *vp = [prepare_hf_dataset(spec, cfg.dataset.cache_dir, tokenizer=cfg.dataset.tokenizer, split=sp)
                         for sp in splits]
        if vp:
            cfg.dataset.validation = {"type": "file", "path": vp[0]}
        cfg.dataset.type, cfg.dataset.path = "file", prepared
    if cfg.dataset.type in ("jsonl", "parquet", "text"):
        from .datasets import prepare_corpus

        if rank == 0:
            prepare_corpus(cfg.dataset.path, cfg.dataset.cache_dir, cfg.dataset.text_field,
                           tokenizer=cfg.dataset.tokenizer)
        if world > 1 and dist.is_initialized():
            dist.barrier()
        prepared = prepare_corpus(cfg.dataset.path, cfg.dataset.cache_dir, cfg.dataset.text_field,
                                  tokenizer=cfg.dataset.tokenizer)
        cfg.dataset.type, cfg.dataset.path = "file", prepared
    vsrc = None
    if cfg.dataset.validation:
        vd = dict(cfg.dataset.validation)
        vtype, vpath = vd.get("type", "file"), vd.get("path")
        if vtype not in ("file", "jsonl", "parquet", "text") or not vpath:
            raise ValueError("dataset.validation needs type = file | jsonl | parquet | text and a path")
        if vtype != "file":
            from .datasets import prepare_corpus

            args = (vpath, vd.get("cache_dir", cfg.dataset.cache_dir), vd.get("text_field", cfg.dataset.text_field))
            if rank == 0:
                prepare_corpus(*args, tokenizer=cfg.dataset.tokenizer)
            if world > 1 and dist.is_initialized():
                dist.barrier()
            vpath = prepare_corpus(*args, tokenizer=cfg.dataset.tokenizer)
        vsrc = (vpath, float(vd.get("train_split_ratio", 0.0)))
    if t.auto_batch_size.enabled:
        from .autotune import choose_batch_size

        res = choose_batch_size(cfg.model, t.block_size, t.auto_batch_size,
                                target_effective_batch=t.target_effective_batch_size)
        t.batch_size = res.batch_size * res.gradient_accumulation_steps
        cfg.parallel.tensor["micro_batches"] = res.gradient_accumulation_steps
        if rank == 0:
            run.write_json("auto_batch_size.json", vars(res))
    ns_path = os.path.join(run.path, "neuron_scaling.json")
    if resume and t.neuron_scaling.enabled and os.path.exists(ns_path):
        import json

        cfg.model.mlp_internal_dim_multiplier = int(json.load(open(ns_path))["mlp_internal_dim_multiplier"])
    if t.epochs is not None:
        t.max_iters = t.epochs * _steps_per_epoch(cfg, 1 if mode in ("tensor_parallel_neuron", "pipeline") else world)
    extended = cfg.model.uses_extended_runtime()
    if not cfg.model.uniform_latent_fanout() and (
            mode not in ("single", "ddp", "fsdp") or t.algorithm == "predictive_coding"
            or t.continual_backprop.enabled or t.neuron_scaling.enabled):
        # as in the reference, local PC needs uniform fan-out; the sharded / pipelined
        # paths and the neuron surgery work on full-width layers
        raise ValueError("model.latent_fanout_schedule needs single / ddp mode without predictive coding, "
                         "continual backprop or neuron scaling")
    if extended and mode not in ("single", "ddp", "fsdp"):
        raise ValueError(f"parallel mode {mode!r} does not support the layer-loop variants this model enables")
    if extended:
        from .runtime_trainer import RuntimeTrainer

        trainer = RuntimeTrainer(cfg.model, dev, lr=o.learning_rate, weight_decay=o.weight_decay,
                                 betas=(o.beta1, o.beta2), eps=o.eps, grad_clip_norm=o.grad_clip_norm,
                                 grad_clip_value=o.grad_clip_value, seed=t.seed,
                                 lr_schedule=o.lr_schedule, max_iters=t.max_iters)
    else:
        trainer = Trainer(cfg.model, dev, lr=o.learning_rate, weight_decay=o.weight_decay,
                          betas=(o.beta1, o.beta2), eps=o.eps, grad_clip_norm=o.grad_clip_norm,
                          grad_clip_value=o.grad_clip_value, seed=t.seed,
                          lr_schedule=o.lr_schedule, max_iters=t.max_iters, comm=comm, tensor_parallel=tp_arg,
                          sequence_parallel=seq_par,
                          micro_batches=micro if mode != "pipeline" else 1)
    runner = None
    if mode == "pipeline":
        from ..parallel.pipeline import PipelineRunner, plan

        pl = plan(cfg.model.n_layer, world, *_pipeline_settings(cfg.parallel.pipeline, world))
        runner = PipelineRunner(trainer.model, pl, rank, t.batch_size // pl.micro, t.block_size)

    pc = t.algorithm == "predictive_coding"
    egg = None
    if o.name == "eggroll" or t.algorithm == "eggroll":
        if extended or pc or mode not in ("single", "ddp", "fsdp") or getattr(trainer, "comm", None) is not None:
            raise ValueError("EGGROLL training needs the plain BDH model in single / ddp mode (NCCL path)")
        o.apply_auto_eggroll_population(t.batch_size)
        egg = o.eggroll_settings()
    if pc and (extended or mode not in ("single", "ddp", "fsdp")):
        raise ValueError("predictive_coding training needs the plain BDH model in single / ddp mode")
    scaler = None
    if t.neuron_scaling.enabled:
        if extended or pc or mode not in ("single", "ddp", "fsdp") or getattr(trainer, "comm", None) is not None:
            raise ValueError("neuron_scaling needs the plain BDH model without the NVLink communicator")
        if not t.validation_interval_iters:
            raise ValueError("neuron_scaling triggers on validation plateaus: set training.validation_interval_iters")
        from .neuron_scaling import NeuronScaler

        scaler = NeuronScaler(t.neuron_scaling)
    mlr = None
    if t.module_lr_scales:
        if extended or mode not in ("single", "ddp", "fsdp") or getattr(trainer, "comm", None) is not None:
            raise ValueError("module_lr_scales needs the plain BDH model without the NVLink communicator")
        from .module_lr import ModuleLrScales

        mlr = ModuleLrScales(t.module_lr_scales, t.max_iters)
    regs = anchor_teacher = None
    if t.logit_entropy_floor.enabled or t.repeat_unlikelihood.enabled or t.dynamics_anchor.enabled \
            or t.greedy_rollout_unlikelihood.enabled:
        t.logit_entropy_floor.validate()
        t.repeat_unlikelihood.validate()
        t.dynamics_anchor.validate()
        t.greedy_rollout_unlikelihood.validate()
        if extended or pc or mode not in ("single", "ddp", "fsdp") or getattr(trainer, "comm", None) is not None:
            raise ValueError("logit_entropy_floor / repeat_unlikelihood need the plain BDH model without the "
                             "NVLink communicator")
        from .logit_regularizers import LogitRegularizers

        regs = LogitRegularizers(t.logit_entropy_floor, t.repeat_unlikelihood, t.dynamics_anchor,
                                 t.greedy_rollout_unlikelihood)
        if t.dynamics_anchor.enabled and t.dynamics_anchor.weight > 0:
            from .objectives import EMATeacher

            anchor_teacher = EMATeacher(trainer.model, min(max(t.dynamics_anchor.teacher_update_rate, 0.0), 1.0))
    objective = None
    if t.objective.get("type", "next_token") != "next_token":
        from . import objectives as OBJ
        from ..config import _fill

        sub = dict(t.objective)
        oc = OBJ.ObjectiveConfig(type=sub.pop("type"),
                                 sdft=_fill(OBJ.SdftObjectiveConfig, sub.pop("sdft", {}), {}, ""),
                                 sdpo=_fill(OBJ.SdpoObjectiveConfig, sub.pop("sdpo", {}), {}, ""),
                                 **{k: v for k, v in sub.items() if k in ("sdft_weight", "sdpo_weight")})
        oc.validate()
        if extended or pc or mode not in ("single", "ddp", "fsdp"):
            raise ValueError("self-distillation objectives need the plain BDH model in single / ddp mode")
        rate = oc.sdpo.teacher_update_rate if oc.type == "sdpo" else oc.sdft.teacher_update_rate
        objective = (oc, OBJ.EMATeacher(trainer.model, rate))
    cbp = None
    if t.continual_backprop.enabled:
        m = cfg.model
        if extended or m.random_scaffold.enabled or mode not in ("single", "ddp", "fsdp"):
            raise ValueError("continual_backprop needs the plain shared low-rank model (no scaffold or "
                             "layer-loop variants) in single / ddp mode")
        from .continual_backprop import ContinualBackprop

        cbp = ContinualBackprop(t.continual_backprop, m, o.learning_rate, seed=t.seed)
    start = 0
    state = None
    if resume and run.latest() is not None:
        info = run.load(t.resume_checkpoint_epoch, trainer.core if extended else trainer.model, trainer.opt,
                        device=dev)
        start = info["step"]
        trainer.step_idx = start
        if hasattr(trainer, "after_load"):
            trainer.after_load()
        if extended and info.get("extra"):
            trainer.load_extra_state(info["extra"])
        rt = info.get("runtime")
        if rt and rt.get("rhos") is not None and not extended:
            state = ModelState(rt["rhos"], int(rt.get("position", 0)))
        elif rt and rt.get("state_tensors") and extended:
            from ..models.dragon_runtime import RuntimeState

            state = RuntimeState.from_tensors(cfg.model.n_layer, rt["state_tensors"], int(rt.get("position", 0)))
    if start == 0 and t.init_checkpoint_path:
        target = trainer.core if extended else trainer.model
        fresh = {n: getattr(target, n).detach().clone() for n in target.store.shapes}
        src = C.RunDir(t.init_checkpoint_path)
        src.load(t.init_checkpoint_epoch, target, None, device=dev)
        if t.init_transfer:
            from ..config import _fill
            from .init_transfer import InitTransferConfig, apply_init_transfer

            apply_init_transfer(target, fresh, _fill(InitTransferConfig, dict(t.init_transfer), {}, ""), device=dev)
    def _teacher():
        for tch in ((objective[1] if objective is not None else None), anchor_teacher,
                    getattr(getattr(trainer, "latent_training", None), "teacher", None)):
            if tch is not None:
                return tch.model
        return None

    if rank == 0:
        from .manifest import write_experiment_manifest

        write_experiment_manifest(cfg, run.path, os.path.basename(os.path.abspath(run.path)), dev.type,
                                  start if start > 0 else None)
    streaming = t.sequence_batching == "streaming" or t.tbptt_persist_across_steps
    if streaming:
        # the stream step (plain, recurrent-state PC or local PC) does not run these
        lost = [name for name, on in (("training.objective", objective is not None),
                                      ("logit regularizers / dynamics anchor / greedy rollout", regs is not None),
                                      ("optimizer.name = eggroll", egg is not None),
                                      ("training.module_lr_scales", mlr is not None),
                                      ("training.neuron_scaling", scaler is not None),
                                      ("training.continual_backprop", cbp is not None)) if on]
        if lost:
            raise ValueError(f"{', '.join(lost)} not implemented with streaming TBPTT batches")
    data_rank = 0 if mode in ("tensor_parallel_neuron", "pipeline") else rank
    data_world = 1 if mode in ("tensor_parallel_neuron", "pipeline") else world
    if mode == "hybrid_2d":
        tp_size = int(cfg.parallel.tensor.get("size", 8))
        data_rank, data_world = rank // tp_size, world // tp_size
    native = None
    if t.native_loader and not streaming:
        try:
            from .native_data import NativeBytes

            if cfg.dataset.type == "file":
                from .datasets import token_bytes

                native = NativeBytes("file", t.batch_size, t.block_size, path=cfg.dataset.path, seed=t.seed,
                                     rank=data_rank, world=data_world, ratio=cfg.dataset.train_split_ratio,
                                     workers=t.loader_workers, start_step=start,
                                     token_bytes=token_bytes(cfg.dataset.path))
            else:
                native = NativeBytes("random", t.batch_size, t.block_size, seed=t.seed, rank=data_rank,
                                     world=data_world, vocab=cfg.model.vocab_size, workers=t.loader_workers,
                                     start_step=start)
        except Exception as e:  # no host toolchain: the Python generators below
            import warnings

            warnings.warn(f"native loader unavailable ({e}); using the Python batch generators", stacklevel=2)
            native = None
    if streaming:
        chunk = t.tbptt_chunk_size or t.block_size
        # a stream (document) is min_logical_block_size tokens rounded up to whole blocks
        doc = -(-max(t.min_logical_block_size or t.block_size, t.block_size) // t.block_size) * t.block_size
        data = StreamingBytes(t.batch_size, doc, chunk, seed=t.seed, rank=data_rank)
        data.pos = (start * chunk) % max(1, t.block_size - chunk + 1) if t.block_size > chunk else 0
    elif cfg.dataset.type == "file" and native is None:
        data = FileBytes(cfg.dataset.path, t.batch_size, t.block_size, "train", cfg.dataset.train_split_ratio,
                         seed=t.seed, rank=data_rank, world=data_world)
        data.step = start
    elif native is not None:
        data = native
    else:
        data = RandomBytes(t.batch_size, t.block_size, seed=t.seed, rank=data_rank, world=data_world)
        data.step = start
    # validation windows: drawn with their own seed (identical across training seeds); a
    # fixed holdout rewinds to the same windows at every validation
    vseed = t.validation.seed % (2**31)
    if vsrc is not None:
        valid = FileBytes(vsrc[0], t.batch_size, t.block_size, "valid", vsrc[1], seed=vseed, rank=data_rank,
                          world=data_world)
    elif cfg.dataset.type == "file":
        valid = FileBytes(cfg.dataset.path, t.batch_size, t.block_size, "valid", cfg.dataset.train_split_ratio,
                          seed=vseed, rank=data_rank, world=data_world)
    else:
        valid = RandomBytes(t.batch_size, t.block_size, seed=vseed, rank=data_rank, world=data_world)
    validate_here = t.validation.execution == "local"
    if t.latent_reasoning.get("enabled"):
        if not (extended and cfg.model.latent_reasoning.enabled):
            raise ValueError("training.latent_reasoning needs model.latent_reasoning.enabled (its JEPA predictor)")
        from .latent_reasoning import LatentReasoningTraining

        trainer.latent_training = LatentReasoningTraining(t.latent_reasoning, cfg.model)
        trainer.latent_training.attach_teacher(trainer.model)
    if start > 0 and _teacher() is not None:
        run.load_teacher(start, _teacher())
    spc = None
    if t.predictive_coding.get("enabled"):
        from .state_pc import RecurrentStatePCConfig

        spc = RecurrentStatePCConfig(**dict(t.predictive_coding))
        spc.validate()
        if not streaming or extended or mode not in ("single", "ddp", "fsdp") \
                or getattr(trainer, "comm", None) is not None:
            raise ValueError("training.predictive_coding (recurrent-state inference) needs streaming TBPTT "
                             "batches on the plain BDH model in single / ddp mode")
    probe = None
    if t.sequence_state_probe.get("enabled"):
        from .state_probe import SequenceStateProbeConfig

        if not streaming or extended:
            raise ValueError("training.sequence_state_probe needs streaming batches on the plain BDH model")
        probe = SequenceStateProbeConfig(**dict(t.sequence_state_probe))

    log = MetricsLogger(run.path, rank, every=t.log_frequency)
    # which step implementation this run takes, and its forward FLOP estimate (the
    # reference logs the same "training path fingerprint" and theoretical profile)
    path = ("pipeline" if runner is not None else mode if mode in ("tensor_parallel_neuron", "hybrid_2d")
            else "runtime_variants" if extended else "predictive_coding" if pc else "eggroll" if egg is not None
            else "self_distillation" if objective is not None
            else "fused_sm100" if getattr(trainer, "fused", False) else "pytorch")
    fl = theoretical_forward_flops(cfg.model, t.batch_size, t.block_size)
    if rank == 0:
        run.write_json("run_info.json", {
            "training_path": path, "world": world, "mode": mode, "comm": comm, "aux_losses": regs is not None,
            "start_step": start, "approx_forward_flops": fl})
    prof = StageProfiler(dev)
    guard = NonFiniteGuard(every=t.log_frequency)
    hb = Heartbeat(timeout=float(os.environ.get("BDH_HEARTBEAT_TIMEOUT", "60"))) if world > 1 else None
    last_loss = None
    step = start
    try:
        for step in range(start, t.max_iters):
            if hb is not None:
                hb.check()
            prof.start("dataloader")
            if streaming:
                x, y, reset = data.next()
                if reset or state is None:
                    if extended:
                        from ..models.dragon_runtime import RuntimeState

                        state = RuntimeState.new(cfg.model.n_layer)
                    else:
                        state = ModelState.empty()
            else:
                x, y = data.next()
            prof.stop("dataloader")
            x_clean = x
            if t.input_corruption.enabled:
                from .corruption import corrupt_inputs

                x = corrupt_inputs(x, t.input_corruption, step, cfg.model.vocab_size, t.seed, rank)
            t0 = time.perf_counter()
            prof.start("forward_backward")
            if runner is not None:
                loss = runner.step(x.to(dev), y.to(dev))
                prof.stop("forward_backward")
                prof.start("optimizer")
                trainer.opt.step()
                trainer.step_idx += 1
                prof.stop("optimizer")
                loss = loss if loss is not None else torch.zeros(())
            elif streaming and pc:
                # layer-local PC on a chunk that continues the carried rho; the state then
                # advances through the chunk with the updated weights, detached
                from .optim import lr_at
                from .predictive_coding import local_pc_step

                xd, yd = x.to(dev), y.to(dev)
                rho0s = None if state.rhos is None else [r.detach() for r in state.rhos]
                loss, _ = local_pc_step(trainer.model, xd, yd, t.local_predictive_coding, rho0s=rho0s)
                trainer.opt.prepare(lr_at(trainer.step_idx, trainer.base_lr, trainer.lr_schedule, trainer.max_iters))
                trainer._update()
                trainer.step_idx += 1
                with torch.no_grad():
                    trainer.model(xd, state=state)
                state.detach_in_place()
                prof.stop("forward_backward")
            elif streaming and spc is not None:
                from .state_pc import state_pc_chunk_loss

                if state.rhos is not None:
                    state.rhos = [r.detach() for r in state.rhos]
                lo, state, _ = state_pc_chunk_loss(trainer.model, x.to(dev), y.to(dev), state, spc, step)
                _autograd_step(trainer, lo)
                state.detach_in_place()
                loss = lo.detach()
                prof.stop("forward_backward")
            elif streaming:
                loss = trainer.step_stream(x, y, state)
                prof.stop("forward_backward")
            elif objective is not None:
                from . import objectives as OBJ

                oc, teacher = objective
                m = trainer.model
                lo = OBJ.window_objective_loss(m, teacher.model, x.to(dev), y.to(dev), oc)
                _autograd_step(trainer, lo)
                teacher.update(m)
                loss = lo.detach()
                prof.stop("forward_backward")
            elif regs is not None and regs.active(step):
                xd, yd = x.to(dev), y.to(dev)
                tl = None
                if anchor_teacher is not None and regs.anchor_active(step):
                    with torch.no_grad():
                        tl = anchor_teacher.model(xd)
                lo = regs.loss(trainer.model(xd), yd, xd, step, teacher_logits=tl, model=trainer.model,
                               clean_inputs=x_clean.to(dev))
                _autograd_step(trainer, lo)
                loss = lo.detach()
                prof.stop("forward_backward")
            elif egg is not None:
                from .eggroll import es_step
                from .optim import lr_at

                lr_now = lr_at(step, o.learning_rate, o.lr_schedule, t.max_iters)
                red = None
                if world > 1:
                    def red(ls):
                        dist.all_reduce(ls)
                        return ls / world
                rep = es_step(trainer.model, x.to(dev), y.to(dev), population=egg["members"] // 2,
                              sigma=egg["sigma"], lr=lr_now, rank=egg["rank"], seed=t.seed * 1_000_003 + step,
                              chunk=None if egg["chunk"] is None else int(egg["chunk"]),
                              weight_decay=o.weight_decay, reduce=red,
                              fitness_normalization=egg["fitness_normalization"],
                              coefficient_clip=egg["coefficient_clip"], max_delta_rms=egg["max_delta_rms"])
                trainer.step_idx += 1
                loss = torch.tensor(rep["mean_loss"])
                prof.stop("forward_backward")
            elif pc:
                from .optim import lr_at
                from .predictive_coding import local_pc_step

                loss, _ = local_pc_step(trainer.model, x.to(dev), y.to(dev), t.local_predictive_coding)
                trainer.opt.prepare(lr_at(trainer.step_idx, trainer.base_lr, trainer.lr_schedule, trainer.max_iters))
                trainer._update()
                trainer.step_idx += 1
                prof.stop("forward_backward")
            else:
                if scaler is not None:
                    scaler.before_step(trainer.model, step)
                if mlr is not None:
                    mlr.before_step(trainer.model, step)
                sample = cbp is not None and cbp.should_sample()
                if sample and not getattr(trainer, "fused", False):
                    cbp.record_reference(trainer.model, x.to(dev))
                loss = trainer.step(x, y)
                if scaler is not None:
                    scaler.after_step(step)
                if mlr is not None:
                    mlr.after_step(step)
                prof.stop("forward_backward")
                if cbp is not None:
                    if sample and getattr(trainer, "fused", False):
                        cbp.record_fused(trainer.model)
                    lr_now = getattr(trainer.opt, "_lr_now", o.learning_rate)
                    if cbp.after_optimizer_step(trainer.model, trainer.opt, lr_now):
                        log.log(step + 1, cbp_replaced=cbp.last.replacement_count, force=True)
            if anchor_teacher is not None:
                anchor_teacher.update(trainer.model)
            if native is not None:
                native.mark_consumed()  # its buffer is refilled only after these copies ran
            prof.tokens += x.numel() * (world if mode in ("ddp", "fsdp") else 1)
            if (step + 1) % t.log_frequency == 0 or step + 1 == t.max_iters:
                lv = float(loss)
                guard.check(0, lv)
                log.log(step + 1, loss=lv, lr=trainer.opt._lr_now if hasattr(trainer.opt, "_lr_now") else o.learning_rate,
                        step_ms=(time.perf_counter() - t0) * 1e3, force=True)
                last_loss = lv
            if validate_here and t.validation_interval_iters and (step + 1) % t.validation_interval_iters == 0 \
                    and runner is None:
                if hasattr(trainer, "sync_params"):
                    trainer.sync_params()  # the PyTorch path reads the full fp32 master
                if probe is not None:
                    from .state_probe import stream_warm_validation

                    chunk_v = t.tbptt_chunk_size or t.block_size
                    vstream = StreamingBytes(t.batch_size, doc, chunk_v, vocab=cfg.model.vocab_size, seed=vseed,
                                             rank=data_rank)
                    rep = stream_warm_validation(trainer.model, vstream, max(doc // chunk_v, 1) * 2, probe, dev)
                    log.log(step + 1, **{f"stream_{k}": v for k, v in rep.items() if k != "state"}, force=True)
                    if rank == 0:
                        run.write_json("sequence_state_probe.json", {"step": step + 1, **rep})
                if t.validation.sampling == "fixed_holdout":
                    valid.step = 0
                vx, vy = valid.next()
                with torch.no_grad():
                    vl = float(trainer.model.loss(vx.to(dev), vy.to(dev)))  # fresh state per window
                log.log(step + 1, valid_loss=vl, force=True)
                if scaler is not None:
                    scaler.observe_validation(vl)
                    if scaler.should_scale(step + 1, trainer.model.cfg):
                        scaler.scale(trainer, step + 1)
                        cfg.model = trainer.model.cfg
                        log.log(step + 1, neuron_scale_event=scaler.events,
                                latent_total=trainer.model.cfg.latent_total, force=True)
                        if rank == 0:
                            run.write_json("neuron_scaling.json", {
                                "mlp_internal_dim_multiplier": trainer.model.cfg.mlp_internal_dim_multiplier,
                                "events": scaler.events, "step": step + 1})
            ck_now = bool(t.checkpoint_interval_iters) and (step + 1) % t.checkpoint_interval_iters == 0
            sharded = ck_now and _save_shards(run, trainer, step + 1, ck_format, extended)
            if ck_now and not sharded and hasattr(trainer, "sync_params"):
                trainer.sync_params()  # every rank: gathers sharded master / moments
            if ck_now and rank == 0:
                rt = None
                if state is not None and not extended and state.rhos is not None:
                    rt = {"position": state.position, "rhos": [r.detach() for r in state.rhos]}
                elif state is not None and extended:
                    rt = {"position": state.position, "state_tensors": state.to_tensors()}
                run.save(step + 1, trainer.core if extended else trainer.model, trainer.opt, {"step": step + 1}, rt,
                         extra=trainer.extra_state() if extended else None, teacher=_teacher(), sharded=sharded)
        sharded = bool(t.checkpoint_interval_iters) and _save_shards(run, trainer, t.max_iters, ck_format, extended)
        if t.checkpoint_interval_iters and not sharded and hasattr(trainer, "sync_params"):
            trainer.sync_params()
        if rank == 0 and t.checkpoint_interval_iters:
            run.save(t.max_iters, trainer.core if extended else trainer.model, trainer.opt, {"step": t.max_iters},
                     extra=trainer.extra_state() if extended else None, teacher=_teacher(), sharded=sharded)
    except PeerFailure:
        if hb is not None:
            hb.stop()
        raise
    finally:
        log.close()
        if native is not None:
            native.close()
        if hb is not None:
            hb.stop()
    summary = prof.summary() if prof.enabled else {}
    run.wait()
    return {"final_loss": last_loss, "steps": t.max_iters - start, "run_dir": run.path, "profile": summary}


def _save_shards(run, trainer, step: int, ck_format: str, extended: bool) -> bool:
    """``sharded_v2``: every data-parallel rank writes its own slices of the fp32 master and
    AdamW moments (no gather); returns True when it did (the other records follow from
    rank 0). Falls back to the unsharded records for trainers without the flat DP layout."""
    if ck_format != "sharded_v2" or extended or not hasattr(trainer, "dp_shard") or trainer.tp is not None:
        return False
    world = trainer.world if trainer.comm is not None else 1
    rank = trainer.comm.rank if trainer.comm is not None else 0
    if trainer.comm is not None or (not dist.is_initialized() or dist.get_rank() == 0):
        slices, master, m, v = trainer.dp_shard()
        run.save_shard(step, rank, world, slices, master, m, v, trainer.model.store.numel, trainer.opt.t)
    if dist.is_initialized():
        dist.barrier()
    return True


def _autograd_step(trainer, loss) -> None:
    """Gradients of ``loss`` by autograd over the PyTorch path of a plain ``BDH``
    model, written into its flat gradient buffer, then the fused AdamW step."""
    from .optim import lr_at

    m = trainer.model
    gr = torch.autograd.grad(loss, list(m.parameters()), allow_unused=True)
    for (n, _), g in zip(m.named_parameters(), gr):
        view = m.store.view(m.store.grad, n)
        view.zero_() if g is None else view.copy_(g)
    trainer.opt.prepare(lr_at(trainer.step_idx, trainer.base_lr, trainer.lr_schedule, trainer.max_iters))
    trainer._update()
    trainer.step_idx += 1


def _steps_per_epoch(cfg: TrainingConfig, data_world: int) -> int:
    """One pass over the train split of a file dataset in [batch, block] windows per
    data-parallel rank; a synthetic stream has no end, so its epoch is the checkpoint
    interval (the reference's fallback, burn_dragon_language/src/train/backend.rs:61-72)."""
    t = cfg.training
    if cfg.dataset.type == "file":
        from .datasets import token_bytes

        n = os.path.getsize(cfg.dataset.path) // token_bytes(cfg.dataset.path)
        train = int(n * cfg.dataset.train_split_ratio)
        return max(1, train // (t.batch_size * t.block_size * max(data_world, 1)))
    return max(1, min(t.checkpoint_interval_iters or t.max_iters, t.max_iters))


def _pipeline_settings(pp: dict, world: int) -> tuple[int, str, int]:
    """(micro-batches, schedule, virtual stages per rank) from ``[parallel.pipeline]``:
    the reference's keys ``microbatches``, ``schedule`` (``gpipe`` | ``interleaved_1f1b``;
    ``1f1b`` also accepted), ``virtual_stages_per_rank`` and ``stage_count``, which must be
    the world size (burn_dragon_train/src/config/core.rs:95-282); ``micro_batches`` is an
    alias of ``microbatches``."""
    micro = int(pp.get("microbatches", pp.get("micro_batches", 4)))
    kind = {"interleaved_1f1b": "interleaved"}.get(pp.get("schedule", "1f1b"), pp.get("schedule", "1f1b"))
    virtual = int(pp.get("virtual_stages_per_rank", 1))
    if "stage_count" in pp and int(pp["stage_count"]) != world:
        raise ValueError(f"parallel.pipeline.stage_count = {pp['stage_count']} but the job has {world} ranks "
                         "(one stage per rank)")
    if micro <= 0 or virtual <= 0:
        raise ValueError("parallel.pipeline.microbatches and virtual_stages_per_rank must be > 0")
    return micro, kind, virtual
