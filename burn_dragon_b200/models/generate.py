"""Generation: batched prefill + recurrent decode with the linear-attention state.

Mirrors the reference's generation paths (burn_dragon_language/src/generation.rs):
``generate_greedy_batch_equal_position`` (:564, batched prefill, then argmax per token on
the device with the host reading a buffer of tokens every ``device_buffer_tokens`` steps,
:650-700) and ``DragonModel::generate`` sampling (temperature / top-k,
burn_dragon_core/src/model/dragon.rs:1729-1811).

On CUDA the prefill runs the fused forward in inference mode (prompt processed in
chunks of ``prefill_chunk`` tokens, the state carried between chunks) and each decode
token runs per layer: x/q = relu(v Dx) with RoPE at the current position (tcgen05
engine, M = batch), the one-pass state update + readout ``rho_step`` kernel, LayerNorm,
the gate GEMM and the split-K decoder GEMM with the fused residual merge. On CPU the
PyTorch path (``models.reference``) does the same with ``ModelState``.
"""

from __future__ import annotations

import math

import torch

from .. import _ext
from ..ops import gemm as G
from ..ops.gemm import Operand
from .reference import rope_freqs
from .state import ModelState


def sample_next(logits: torch.Tensor, temperature: float = 0.0, top_k: int | None = None,
                generator: torch.Generator | None = None) -> torch.Tensor:
    """Greedy for temperature 0, else softmax(logits / T) restricted to the top-k."""
    if temperature <= 0.0:
        return logits.argmax(dim=-1)
    z = logits.float() / temperature
    if top_k is not None and top_k < z.shape[-1]:
        kth = torch.topk(z, top_k, dim=-1).values[..., -1:]
        z = z.masked_fill(z < kth, float("-inf"))
    p = torch.softmax(z, dim=-1)
    return torch.multinomial(p, 1, generator=generator).squeeze(-1)


class _DecodeWorkspace:
    def __init__(self, cfg, B: int, device):
        D, H, Nh, V = cfg.n_embd, cfg.n_head, cfg.latent_per_head, cfg.vocab_size
        N = H * Nh
        f32, bf16 = torch.float32, torch.bfloat16
        e = lambda *s, dt=f32: torch.empty(*s, dtype=dt, device=device)  # noqa: E731
        self.B = B
        self.v32 = [e(B, D), e(B, D)]
        self.v16 = [e(B, D, dt=bf16), e(B, D, dt=bf16)]
        self.x16, self.q16 = e(B, N, dt=bf16), e(B, N, dt=bf16)
        self.a32 = e(B, H, D)
        self.amean, self.arstd = e(B * H), e(B * H)
        self.an16 = e(B, H, D, dt=bf16)
        self.yn16 = e(B, N, dt=bf16)
        kb = N // 64
        self.splits = G.fit_splits(kb, max(1, 148 // max(1, -(-B // 128))))
        self.partial = e(self.splits, B, D)
        self.emb = e(B, D)
        self.logits = e(B, V)
        self.freq = rope_freqs(Nh, cfg.rope_theta, device=device) if cfg.rotary_embedding == "rope" else None
        self.gamma = None
        if cfg.uses_decay():
            self.gamma = torch.exp(-torch.tensor(cfg.decay_slopes(), dtype=torch.float64)).float().to(device)


class Generator:
    def __init__(self, model, prefill_chunk: int = 512, state_dtype: str = "fp32"):
        """``state_dtype`` "bf16": the decode steps keep the recurrent state rho in bf16
        (half the state traffic, which is the whole cost of a decode token; each update is
        computed in fp32 and rounded once when stored). The prefill still builds the state
        in fp32; it is rounded to bf16 at the first decode step."""
        if state_dtype not in ("fp32", "bf16"):
            raise ValueError("state_dtype must be 'fp32' or 'bf16'")
        self.state_dtype = state_dtype
        self.model = model
        self.cfg = model.cfg
        self.prefill_chunk = prefill_chunk
        self._dws: _DecodeWorkspace | None = None
        self._pws = None
        from .bdh_fused import fused_unsupported

        # options the fused prefill / decode kernels do not implement run on the PyTorch path
        self._fused_ok = fused_unsupported(self.cfg) is None

    # ---------------------------------------------------------------- prefill
    @torch.no_grad()
    def prefill(self, prompt: torch.Tensor, state: ModelState | None = None) -> tuple[torch.Tensor, ModelState]:
        """Run the prompt [B, T] through the model; returns (last-position logits [B, V], state)."""
        state = state or ModelState.empty()
        B, T = prompt.shape
        dev = prompt.device
        fused_ok = dev.type == "cuda" and self._fused_ok
        chunk = self.prefill_chunk if fused_ok else T
        main = (T // 128) * 128 if fused_ok else 0
        if fused_ok and 0 < main < T:
            # the fused prefill takes whole 128-token blocks; the tail runs as decode steps
            logits, state = self.prefill(prompt[:, :main], state)
            for t in range(main, T):
                logits = self.decode_step(prompt[:, t].contiguous(), state)
            return logits, state
        if fused_ok and main:
            chunk = math.gcd(main, chunk) if chunk % 128 == 0 else 128
        if not fused_ok or main == 0:
            if not fused_ok:
                logits = self.model(prompt, state=state)
                state.detach_in_place()
                return logits[:, -1].float(), state
            logits = None
            for t in range(T):
                logits = self.decode_step(prompt[:, t].contiguous(), state)
            return logits, state
        from .bdh_fused import FusedBDH, FusedWorkspace

        if self._pws is None or self._pws.B != B or self._pws.T != chunk:
            self._pws = None
            torch.cuda.empty_cache()
            self._pws = FusedWorkspace(self.cfg, B, chunk, dev, inference=True)
        f = FusedBDH(self.cfg, self._pws)
        p32 = self.model.store.views(self.model.store.data)
        p16 = self.model.shadow_dict()
        for s in range(0, T, chunk):
            rho0s = state.rhos
            if rho0s is not None and rho0s[0].dtype != torch.float32:
                rho0s = [r.float() for r in rho0s]  # the prefill carries its state in fp32
            outs = f.forward(p16, p32, prompt[:, s:s + chunk], pos0=state.position, rho0s=rho0s,
                             want_state=True)
            state.rhos = outs
            state.position += chunk
        logits = self._pws.logits.view(B, chunk, -1)[:, -1].clone()
        return logits, state

    # ---------------------------------------------------------------- decode
    @torch.no_grad()
    def decode_step(self, tokens: torch.Tensor, state: ModelState) -> torch.Tensor:
        """One token per sequence: tokens [B] -> logits [B, V]; advances ``state``."""
        if tokens.device.type != "cuda" or not self._fused_ok:
            logits = self.model(tokens[:, None], state=state)
            state.detach_in_place()
            return logits[:, -1].float()
        cfg = self.cfg
        tokens = tokens.contiguous()
        B = tokens.shape[0]
        if self._dws is None or self._dws.B != B:
            self._dws = _DecodeWorkspace(cfg, B, tokens.device)
        w = self._dws
        mod = _ext.load()
        D, H, Nh, V = cfg.n_embd, cfg.n_head, cfg.latent_per_head, cfg.vocab_size
        N = H * Nh
        p32 = self.model.store.views(self.model.store.data)
        p16 = self.model.shadow_dict()
        gam, bet, eps = p32["norm_gamma"], p32["norm_beta"], cfg.norm_eps
        from .bdh_fused import norm_kwargs

        nk = norm_kwargs(cfg, p32)
        thr, thr_y = cfg.thresholds()
        sdt = torch.bfloat16 if self.state_dtype == "bf16" else torch.float32
        if state.rhos is None:
            state.rhos = [torch.zeros(B, H, Nh, D, device=tokens.device, dtype=sdt) for _ in range(cfg.n_layer)]
        elif state.rhos[0].dtype != sdt:
            state.rhos = [r.to(sdt) for r in state.rhos]
        mod.ln_fwd(p32["embed"], tokens, B, D, gam, bet, eps, w.v32[0], w.v16[0], w.amean, w.arstd, **nk)
        B_enc = Operand(p16["encoder"], True, Nh, D, Nh, z1=(H, D * Nh))
        B_encv = Operand(p16["encoder_v"], True, Nh, D, Nh, z1=(H, D * Nh))
        cur = 0
        for l in range(cfg.n_layer):
            v32, v16 = w.v32[cur], w.v16[cur]
            G.gemm(G.EPI_RELU_ROPE, Operand(v16, False, D, B, D), B_enc, B, Nh, D, w.x16, Z1=H, bn=128,
                   out1=w.q16 if w.freq is not None else None, ld=N, sz1=Nh, thr=thr, freq=w.freq, T=1,
                   pos0=state.position, Nh=Nh)
            q = w.q16 if w.freq is not None else w.x16
            w.a32.zero_()
            mod.rho_step(state.rhos[l], q, N, v32, w.gamma, w.a32, B, H, Nh, D)
            mod.ln_fwd(w.a32, None, B * H, D, gam, bet, eps, None, w.an16, w.amean, w.arstd, **nk)
            G.gemm(G.EPI_GATE, Operand(w.an16, False, D, B, H * D, z1=(H, D)), B_encv, B, Nh, D, w.yn16, Z1=H,
                   bn=128, aux0=w.x16, ld=N, sz1=Nh, thr=thr_y)
            G.gemm(G.EPI_F32, Operand(w.yn16, False, N, B, N), Operand(p16["decoder"], True, D, N, D), B, D, N,
                   w.partial, splits=w.splits, ld=D, split_stride=B * D)
            nxt = 1 - cur
            mod.tail_fwd(w.partial, w.splits, B * D, v32, B, D, gam, bet, eps, None, w.v32[nxt], w.v16[nxt], None, **nk)
            cur = nxt
        G.gemm(G.EPI_F32, Operand(w.v16[cur], False, D, B, D), Operand(p16["lm_head"], True, V, D, V), B, V, D,
               w.logits, ld=V)
        state.position += 1
        return w.logits

    # ---------------------------------------------------------------- ragged batches
    @torch.no_grad()
    def generate_ragged(self, prompts: list[list[int]], max_new_tokens: list[int], stop_token: int | None = None,
                        device_buffer_tokens: int = 64, device=None) -> list[list[int]]:
        """Exact greedy continuations of prompts of different lengths in one batch
        (burn_dragon_language/src/generation.rs:296-560): every row advances at the same
        absolute position; a row still inside its prompt consumes its next prompt token,
        a finished one its argmax. Tokens stay on the device for ``device_buffer_tokens``
        steps; the host then applies budgets and the stop token (kept in the output)
        and drops finished rows from the batch (the recurrent state is row-separable)."""
        if len(prompts) != len(max_new_tokens):
            raise ValueError("one token budget per prompt")
        if any(len(p) == 0 for p in prompts):
            raise ValueError("prompts must be non-empty")
        dev = torch.device(device) if device is not None else self.model.store.data.device
        out: list[list[int]] = [[] for _ in prompts]
        rows = [r for r, b in enumerate(max_new_tokens) if b > 0]
        if not rows:
            return out
        lens = torch.tensor([len(prompts[r]) for r in rows], device=dev)
        width = int(lens.max())
        table = torch.zeros(len(rows), width, dtype=torch.long, device=dev)
        for i, r in enumerate(rows):
            table[i, :len(prompts[r])] = torch.tensor(prompts[r], device=dev)
        shared = int(lens.min())
        logits, state = self.prefill(table[:, :shared].contiguous())
        nbuf = max(1, device_buffer_tokens)
        while rows:
            toks = torch.empty(len(rows), nbuf, dtype=torch.long, device=dev)
            gen = torch.empty(len(rows), nbuf, dtype=torch.bool, device=dev)
            for k in range(nbuf):
                pos = state.position
                in_prompt = lens > pos
                prompt_tok = table[:, min(pos, width - 1)]
                nxt = torch.where(in_prompt, prompt_tok, logits.argmax(-1))
                toks[:, k] = nxt
                gen[:, k] = ~in_prompt
                logits = self.decode_step(nxt.contiguous(), state)
            host_t, host_g = toks.cpu().tolist(), gen.cpu().tolist()
            keep = []
            for i, r in enumerate(rows):
                stopped = False
                for t, g in zip(host_t[i], host_g[i]):
                    if not g or len(out[r]) >= max_new_tokens[r]:
                        continue
                    out[r].append(t)
                    if stop_token is not None and t == stop_token:
                        stopped = True
                        break
                if not stopped and len(out[r]) < max_new_tokens[r]:
                    keep.append(i)
            if len(keep) < len(rows):
                idx = torch.tensor(keep, device=dev, dtype=torch.long)
                rows = [rows[i] for i in keep]
                if not rows:
                    break
                state.rhos = [r_.index_select(0, idx).contiguous() for r_ in state.rhos]
                lens, table, logits = lens[idx], table[idx], logits[idx]
        return out

    # ---------------------------------------------------------------- streaming
    @torch.no_grad()
    def generate_stream(self, prompt: list[int], max_new_tokens: int, chunk_tokens: int = 16,
                        temperature: float = 0.0, top_k: int | None = None, stop_token: int | None = None,
                        sliding_window: int | None = None, on_chunk=None, seed: int | None = None,
                        device=None) -> list[int]:
        """One sequence, tokens handed to ``on_chunk`` every ``chunk_tokens`` steps
        (generation.rs:1174-1275). ``sliding_window`` keeps only the last ``window``
        prompt tokens (the recurrent state needs no trimming afterwards)."""
        dev = torch.device(device) if device is not None else self.model.store.data.device
        if sliding_window and len(prompt) > sliding_window:
            prompt = prompt[-sliding_window:]
        gen = None
        if seed is not None:
            gen = torch.Generator(device=dev)
            gen.manual_seed(seed)
        logits, state = self.prefill(torch.tensor([prompt], device=dev))
        full = list(prompt)
        pending = []
        done = 0
        while done < max_new_tokens:
            nxt = sample_next(logits, temperature, top_k, gen)
            pending.append(nxt)
            done += 1
            if done < max_new_tokens:
                logits = self.decode_step(nxt.contiguous(), state)
            if len(pending) >= chunk_tokens or done == max_new_tokens:
                chunk = torch.cat(pending).cpu().tolist()
                pending.clear()
                if stop_token is not None and stop_token in chunk:
                    chunk = chunk[:chunk.index(stop_token) + 1]
                    full.extend(chunk)
                    if on_chunk:
                        on_chunk(chunk)
                    break
                full.extend(chunk)
                if on_chunk:
                    on_chunk(chunk)
        return full

    # ---------------------------------------------------------------- loop
    @torch.no_grad()
    def generate(self, prompt: torch.Tensor, max_new_tokens: int, temperature: float = 0.0,
                 top_k: int | None = None, device_buffer_tokens: int = 64, seed: int | None = None):
        """Returns [B, max_new_tokens] generated tokens (host tensor)."""
        gen = None
        if seed is not None:
            gen = torch.Generator(device=prompt.device)
            gen.manual_seed(seed)
        logits, state = self.prefill(prompt)
        buf = torch.empty(prompt.shape[0], max_new_tokens, dtype=torch.long, device=prompt.device)
        out = []
        nxt = sample_next(logits, temperature, top_k, gen)
        for i in range(max_new_tokens):
            buf[:, i] = nxt
            if (i + 1) % device_buffer_tokens == 0 or i + 1 == max_new_tokens:
                start = (i // device_buffer_tokens) * device_buffer_tokens
                out.append(buf[:, start:i + 1].cpu())
            if i + 1 < max_new_tokens:
                logits = self.decode_step(nxt, state)
                nxt = sample_next(logits, temperature, top_k, gen)
        return torch.cat(out, dim=1)
