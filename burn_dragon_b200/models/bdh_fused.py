"""The BDH training step on the sm_100a kernels: forward, loss and hand-written backward.

Every contraction of the shared-weight layer stack runs on the tcgen05 engine with its
elementwise work fused into the epilogue; the row-wise LayerNorm / residual-merge /
cross-entropy work runs in one-warp-per-row kernels. Activations of every layer are
kept resident in HBM (about 3.4 GB per layer at BDH-GPU batch 32 x 512), so the backward
recomputes nothing.

Layouts (M = B*T token rows, N = H*Nh neurons):
  v      [M, D]     fp32 residual stream (+ bf16 copy as GEMM operand)
  x, q   [M, N]     bf16 relu(v Dx) and rope(x)  (column = h*Nh + j)
  S      [B,H,T,T]  bf16 strictly-causal scores q q^T (zeros on and above the diagonal)
  a      [M, H, D]  fp32 attention output before its LayerNorm; an = LN(a) in bf16
  yn     [M, N]     bf16 x * relu(an Dy)
Parameters keep the reference layouts: encoder / encoder_v [H, D, Nh], decoder [N, D],
embed [V, D], lm_head [D, V] (burn_dragon_core/src/model/dragon.rs:240-272).

Reference call stack mirrored: dragon/language_pipeline.rs:55-411 (embedding LN, layer
loop), dragon/residual_stream.rs:323-572 (layer), dragon/language_head.rs:549-572 (CE).
"""

from __future__ import annotations

import math
import os

import torch

from .. import _ext
from ..ops import gemm as G
from ..ops.gemm import Operand
from .reference import rope_freqs

# The forward stores x = relu(v Dx) next to q = rope(x) (the gate and the decoder
# backward read x); the step roofline counts its bytes.
STORES_X = True
# RoPE phases from a half2 (cos, sin) table instead of evaluating them in the epilogue:
# BDH_ROPE_TMA=1 stages the x-projection's table tiles through its epilogue's TMA ring,
# BDH_ROPE_TABLE=1 has dQ read them with plain loads. Both off by default: at BDH-GPU batch
# 32 the staged table took the x-projection from 597 to 765 us (the two-buffer ring must
# drain a tile's stores before the next table tile may land) and the plain loads expose
# their latency.
ROPE_TABLE = os.environ.get("BDH_ROPE_TABLE", "0") == "1"
ROPE_TMA = os.environ.get("BDH_ROPE_TMA", "0") == "1"


# Vocabularies up to this size take the scan form of the embedding-gradient kernel
# (every block reads the token list); larger ones walk a stable token sort.
EMBED_SCAN_MAX_V = 1024


def embed_grad(mod, tokens: torch.Tensor, rows_grad: torch.Tensor, table_grad: torch.Tensor,
               accumulate: bool) -> None:
    """table_grad[v] (+)= sum of rows_grad[r] over rows with tokens[r] == v, in row order
    (deterministic: no atomics). ``tokens`` int64 [R], ``rows_grad`` fp32 [R, D]."""
    tok = tokens.reshape(-1)
    if tok.dtype != torch.int64 or not tok.is_contiguous():
        tok = tok.to(torch.int64).contiguous()
    R, D = rows_grad.shape
    V = table_grad.shape[0]
    if V <= EMBED_SCAN_MAX_V:
        mod.embed_grad(tok, rows_grad, R, D, table_grad, accumulate, None, None)
        return
    srt, perm = torch.sort(tok, stable=True)
    seg = torch.searchsorted(srt, torch.arange(V + 1, device=tok.device, dtype=torch.int64))
    mod.embed_grad(tok, rows_grad, R, D, table_grad, accumulate, perm, seg)


# Norm kinds of the row kernels (rowwise.cu NormArgs).
NORM_KINDS = {"layer_norm": 0, "rms_norm": 1, "dynamic_tanh": 2, "derf": 3}


def norm_kwargs(cfg, p32: dict) -> dict:
    """The trailing norm arguments of the row kernels: the kind and, for the elementwise
    kinds, the learnable alpha / shift scalars (1-element fp32 device tensors)."""
    k = NORM_KINDS[getattr(cfg, "norm_kind", "layer_norm")]
    return {"norm_kind": k, "norm_alpha": p32.get("norm_alpha") if k >= 2 else None,
            "norm_shift": p32.get("norm_shift") if k == 3 else None}


def fused_unsupported(cfg) -> str | None:
    """The first model option the fused kernels do not implement, or None: they
    implement dropout 0 (as the BDH-GPU profiles use), every norm kind (LayerNorm, RMSNorm,
    DynamicTanh, Derf), RoPE / ALiBi / no rotation, one residual stream and an untied
    output head."""
    if cfg.dropout != 0.0:
        return "dropout > 0"
    if getattr(cfg, "norm_kind", "layer_norm") not in NORM_KINDS:
        return f"norm_kind {cfg.norm_kind!r}"
    if cfg.rotary_embedding == "pope":
        return "PoPE"
    if getattr(cfg, "mhc_streams", 1) > 1:
        return "mHC streams"
    if cfg.tie_input_output_embeddings:
        return "a tied lm_head"
    if getattr(cfg, "latent_fanout_schedule", None) and not cfg.uniform_latent_fanout():
        return "a latent fan-out schedule"
    rs = getattr(cfg, "random_scaffold", None)
    if rs is not None and rs.enabled and rs.rank not in (4, 8, 16, 32):
        return f"random-scaffold rank {rs.rank} (the adapter-gradient kernel has ranks 4, 8, 16, 32)"
    return None


class FusedWorkspace:
    """Activation and gradient buffers for one (B, T) shape, allocated once."""

    def __init__(self, cfg, B: int, T: int, device: torch.device, inference: bool = False):
        """``inference``: forward-only workspace (one set of per-layer activation buffers
        reused by every layer, outgoing state written in place over the incoming one)."""
        self.cfg = cfg
        self.inference = inference
        self.B, self.T = B, T
        D, H, Nh, V = cfg.n_embd, cfg.n_head, cfg.latent_per_head, cfg.vocab_size
        N, M, L = H * Nh, B * T, cfg.n_layer
        self.D, self.H, self.Nh, self.N, self.M, self.L, self.V = D, H, Nh, N, M, L, V
        if T % 128 or M % 128 or Nh % 64 or D % 32 or V % 32:
            raise ValueError("fused BDH path needs T % 128 == 0, Nh % 64 == 0, D % 32 == 0, V % 32 == 0")
        dev = device
        f32, bf16 = torch.float32, torch.bfloat16
        e = lambda *s, dt=f32: torch.empty(*s, dtype=dt, device=dev)  # noqa: E731
        def per_layer(make, count=L):
            if inference:
                one = make()
                return [one] * count
            return [make() for _ in range(count)]

        self.v32 = per_layer(lambda: e(M, D), L + 1) if not inference else [e(M, D), e(M, D)] * (L // 2 + 1)
        self.v16 = per_layer(lambda: e(M, D, dt=bf16), L + 1) if not inference else \
            [e(M, D, dt=bf16), e(M, D, dt=bf16)] * (L // 2 + 1)
        self.x16 = per_layer(lambda: e(M, N, dt=bf16))
        self.q16 = per_layer(lambda: e(M, N, dt=bf16)) if cfg.rotary_embedding == "rope" else self.x16
        self.S16 = per_layer(lambda: e(B, H, T, T, dt=bf16))
        self.a32 = per_layer(lambda: e(M, H, D))
        self.amean = per_layer(lambda: e(M * H))
        self.arstd = per_layer(lambda: e(M * H))
        self.an16 = per_layer(lambda: e(M, H, D, dt=bf16))
        self.yn16 = per_layer(lambda: e(M, N, dt=bf16))
        self.m32 = per_layer(lambda: e(M, D))
        self.tst = per_layer(lambda: e(M, 4))
        self._tok = None
        self.emean, self.erstd = e(M), e(M)
        self.logits = e(M, V)
        self.dlogits16 = e(M, V, dt=bf16)
        self.loss_rows = e(M)
        self.inv_count = torch.full((1,), 1.0 / M, dtype=f32, device=dev)
        # split-K for the decoder product (K = N is long, only M/128 output tiles)
        kb = -(-N // 64)
        tiles = -(-M // 128) * -(-D // G.pick_bn(D))
        self.dec_splits = G.fit_splits(kb, max(1, -(-2 * 148 // tiles)))
        self.partial = e(self.dec_splits, M, D)
        if inference:
            self.rho16 = None
            self.rho_sets = None
            self.rho16_sets = None
            self.rho16_valid = [False, False]
            self.rho_flip = 0
            self.has_rho0 = False
            self.qscaled = None
            self.freq = rope_freqs(Nh, cfg.rope_theta, device=dev) if cfg.rotary_embedding == "rope" else None
            self.log2_decay = None
            if cfg.uses_decay():
                g = torch.tensor(cfg.decay_slopes(), dtype=torch.float64)
                self.log2_decay = (-g / math.log(2.0)).to(torch.float32).to(dev)
            return
        # backward temporaries (shared across layers)
        self.dx16 = e(M, N, dt=bf16)
        self.dy16 = e(M, N, dt=bf16)
        self.dm16 = e(M, D, dt=bf16)
        self.dv_res = e(M, D)
        self.dan32 = e(M, H, D)
        self.dC16 = e(B, H, T, D, dt=bf16)
        self.P32 = e(B, H, T, T)
        self.G16 = e(B, H, T, T, dt=bf16)
        self.dva32 = e(M, D)
        self.dvx32 = e(H, M, D)
        self.dv = [e(M, D), e(M, D)]
        self.freq = rope_freqs(Nh, cfg.rope_theta, device=dev) if cfg.rotary_embedding == "rope" else None
        if cfg.uses_decay():
            g = torch.tensor(cfg.decay_slopes(), dtype=torch.float64)
            self.log2_decay = (-g / math.log(2.0)).to(torch.float32).to(dev)  # log2(exp(-s))
        else:
            self.log2_decay = None
        # stateful (TBPTT / streaming) buffers, allocated on first use: the bf16 operand
        # copy of the incoming state and two ping-pong sets of outgoing fp32 states
        self.rho16: list[torch.Tensor] | None = None
        self.rho_sets: list[list[torch.Tensor]] | None = None
        self.rho16_sets: list[list[torch.Tensor]] | None = None
        self.rho16_valid = [False, False]
        self.rho_flip = 0
        self.has_rho0 = False
        self.qscaled: torch.Tensor | None = None

    def token_ids(self, tokens: torch.Tensor) -> torch.Tensor:
        """The step's token ids as a flat contiguous int64 tensor (the caller's tensor when it
        already is one, else a copy into a workspace buffer, so a captured graph keeps one
        address)."""
        t = tokens.reshape(-1)
        if t.dtype == torch.int64 and t.is_contiguous():
            return t
        if self._tok is None or self._tok.numel() != t.numel():
            self._tok = torch.empty(t.numel(), dtype=torch.int64, device=t.device)
        self._tok.copy_(t)
        return self._tok

    def rope_tab(self, pos0: int, staged: bool = False):
        """The half2 (cos, sin) table of this workspace's positions pos0 .. pos0 + T - 1
        (rebuilt only when pos0 changes), or None without RoPE. ``staged``: for the
        x-projection, which fetches table tiles by TMA (only with BDH_ROPE_TMA=1); else for
        dQ's plain loads (only with BDH_ROPE_TABLE=1)."""
        if self.freq is None or not (ROPE_TMA if staged else ROPE_TABLE):
            return None
        if getattr(self, "_rope_tab", None) is None:
            self._rope_tab = torch.empty(self.T, self.Nh // 2, dtype=torch.int32, device=self.freq.device)
            self._rope_pos0 = None
        if self._rope_pos0 != pos0:
            G.rope_table(self.freq, pos0, self.T, self._rope_tab)
            self._rope_pos0 = pos0
        return self._rope_tab

    def ensure_state_buffers(self) -> None:
        """Training: two ping-pong sets of outgoing fp32 states with their bf16 operand
        copies (written by the state GEMM's epilogue, so the next chunk reads its incoming
        state as a GEMM operand without a conversion pass). Inference: one bf16 operand
        buffer, the outgoing state overwriting the incoming one."""
        if self.rho16 is not None:
            return
        B, H, Nh, D, L = self.B, self.H, self.Nh, self.D, self.L
        dev = self.v32[0].device
        if self.inference:
            one16 = torch.empty(B, H, Nh, D, dtype=torch.bfloat16, device=dev)
            self.rho16 = [one16] * L
            self.rho_sets = None
            self.rho16_sets = None
        else:
            self.rho_sets = [[torch.empty(B, H, Nh, D, dtype=torch.float32, device=dev) for _ in range(L)]
                             for _ in range(2)]
            self.rho16_sets = [[torch.empty(B, H, Nh, D, dtype=torch.bfloat16, device=dev) for _ in range(L)]
                               for _ in range(2)]
            self.rho16 = list(self.rho16_sets[0])
        self.rho16_valid = [False, False]


def _bn(n: int) -> int:
    return G.pick_bn(n)


class FusedBDH:
    """Runs forward + CE + backward of the BDH stack for a fixed workspace."""

    def __init__(self, cfg, ws: FusedWorkspace, tp=None):
        """``tp``: optional ``parallel.tp.TensorParallel``; the workspace then holds this
        rank's heads only and the decoder / residual-gradient partials are summed over
        the tensor-parallel group."""
        self.tp = tp
        why = fused_unsupported(cfg)
        if why is not None:
            raise ValueError(f"the fused path does not implement {why} (use the PyTorch path)")
        self.cfg = cfg
        self.ws = ws
        self.mod = _ext.load()
        G.error_word(ws.v32[0].device)  # (registers the bounds-check word under DRAGON_DEBUG_BOUNDS=1)

    # ---------------------------------------------------------------- forward
    def forward(self, p16: dict, p32: dict, tokens: torch.Tensor | None, pos0: int = 0, rho0s=None,
                want_state: bool = False, v_in: torch.Tensor | None = None, with_head: bool = True):
        """Forward of the stack. With ``rho0s`` (per-layer fp32 [B,H,Nh,D]) the carried
        linear-attention state enters every layer (C += gamma^t q rho0); with
        ``want_state`` the per-layer final states are returned (fp32, owned by the
        workspace: valid until the step after next).

        Pipeline stages: ``v_in`` ([M, D] fp32) replaces the embedding (a later stage),
        ``with_head=False`` stops after this stage's layers (the output is ``ws.v32[L]``)."""
        ws, cfg, mod = self.ws, self.cfg, self.mod
        decay = ws.log2_decay is not None
        ws.has_rho0 = rho0s is not None
        out_states = None
        out16 = None
        in16 = None  # bf16 operand copies of the incoming states, when a state GEMM wrote them
        if rho0s is not None or want_state:
            ws.ensure_state_buffers()
        if not ws.inference and ws.rho_sets is not None:
            cur = ws.rho_flip
            prev = cur ^ 1
            if rho0s is not None:
                if ws.rho16_valid[prev] and all(r.data_ptr() == s.data_ptr() for r, s in zip(rho0s, ws.rho_sets[prev])):
                    in16 = ws.rho16_sets[prev]
                else:
                    # a state from elsewhere (checkpoint, probe): its operand copy goes into the
                    # set this step does not write
                    for l in range(ws.L):
                        ws.rho16_sets[prev][l].copy_(rho0s[l])
                    ws.rho16_valid[prev] = False
                    in16 = ws.rho16_sets[prev]
                ws.rho16 = list(in16)
        if want_state:
            if ws.inference:
                if rho0s is None:
                    rho0s_buf = [torch.empty(ws.B, ws.H, ws.Nh, ws.D, device=ws.v32[0].device) for _ in range(ws.L)]
                    out_states = rho0s_buf
                else:
                    out_states = list(rho0s)  # updated in place
            else:
                out_states = ws.rho_sets[ws.rho_flip]
                out16 = ws.rho16_sets[ws.rho_flip]
                ws.rho16_valid[ws.rho_flip] = True
                ws.rho_flip ^= 1
        elif not ws.inference and ws.rho_sets is not None:
            ws.rho16_valid = [False, False]
        B, T, D, H, Nh, N, M, L = ws.B, ws.T, ws.D, ws.H, ws.Nh, ws.N, ws.M, ws.L
        peer = None
        if self.tp is not None and self.tp.world > 1 and not ws.inference:
            peer = self.tp.attach_peer(M, D, L, ws.v32[0].device)
            if peer is not None and self.tp.sequence_parallel:
                # sequence parallel: the bf16 residual operands and the bf16 decoder
                # gradient live in symmetric memory (rows gathered from their owners)
                ws.v16 = peer.v16_views
                ws.dm16 = peer.dm16
            elif peer is not None:
                ws.m32 = peer.sum_views  # the all-gathered decoder sums land here
        eps = cfg.norm_eps
        nk = norm_kwargs(cfg, p32)
        thr, thr_y = cfg.thresholds()
        if v_in is None:
            # the embedding rows are gathered inside the norm kernel (and again in its backward)
            tok = ws.token_ids(tokens)
            mod.ln_fwd(p32["embed"], tok, M, D, p32["norm_gamma"], p32["norm_beta"], eps, ws.v32[0], ws.v16[0],
                       ws.emean, ws.erstd, **nk)
        else:
            ws.v32[0].copy_(v_in.reshape(M, D))
            ws.v16[0].copy_(ws.v32[0])
        enc, encv, dec = p16["encoder"], p16["encoder_v"], p16["decoder"]
        B_enc = Operand(enc, True, Nh, D, Nh, z1=(H, D * Nh))
        B_encv = Operand(encv, True, Nh, D, Nh, z1=(H, D * Nh))
        B_dec = Operand(dec, True, D, N, D)
        for l in range(L):
            v16 = ws.v16[l]
            # x = relu(v Dx - thr), q = rope(x)       (K = D)
            G.gemm(G.EPI_RELU_ROPE, Operand(v16, False, D, M, D), B_enc, M, Nh, D, ws.x16[l], Z1=H, bn=G.tma_bn(M, Nh),
                   out1=ws.q16[l] if ws.freq is not None else None, ld=N, sz1=Nh, thr=thr, freq=ws.freq,
                   T=T, pos0=pos0, Nh=Nh, rope_tab=ws.rope_tab(pos0, staged=True))
            # S = tril_{-1}(q q^T) (* gamma^(i-j))      (K = Nh), upper tiles skipped
            qop = Operand(ws.q16[l], False, Nh, T, N, z1=(H, Nh), z2=(B, T * N))
            # 256-row CTA-pair tiles x 128 columns: finer causal skipping than 256 x 256
            # (6 of 8 tiles vs 3 of 4 at T = 512), 8% faster measured at BDH-GPU batch 32
            G.gemm(G.EPI_SCORES, qop, qop, T, T, Nh, ws.S16[l], Z1=H, Z2=B, bn=128,
                   causal_skip=True, ld=T, sz1=T * T, sz2=H * T * T, log2_decay=ws.log2_decay)
            # a = S V                                   (K = T), V shared by the heads
            G.gemm(G.EPI_F32, Operand(ws.S16[l], False, T, T, T, z1=(H, T * T), z2=(B, H * T * T)),
                   Operand(v16, True, D, T, D, z2=(B, T * D)), T, D, T, ws.a32[l], Z1=H, Z2=B,
                   ld=H * D, sz1=D, sz2=T * H * D)
            if rho0s is not None:
                # a += gamma^t q rho0                    (K = Nh)
                if in16 is None:
                    ws.rho16[l].copy_(rho0s[l])
                G.gemm(G.EPI_F32, qop, Operand(ws.rho16[l], True, D, Nh, D, z1=(H, Nh * D), z2=(B, H * Nh * D)),
                       T, D, Nh, ws.a32[l], Z1=H, Z2=B, ld=H * D, sz1=D, sz2=T * H * D, accumulate=True,
                       log2_decay=ws.log2_decay, row_decay=decay)
            if want_state:
                # rho_T = gamma^T rho0 + (q * gamma^(T-t))^T v      (K = T)
                ro = out_states[l]
                qsrc = ws.q16[l]
                if decay:
                    g = torch.exp2(ws.log2_decay.double())  # gamma per head
                    tt = torch.arange(T, device=ro.device, dtype=torch.float64)
                    sc = (g[None, :] ** (T - tt)[:, None]).float()  # [T, H]
                    if ws.qscaled is None:
                        ws.qscaled = torch.empty_like(ws.q16[l])
                    qv = ws.q16[l].view(B, T, H, Nh).float() * sc[None, :, :, None]
                    ws.qscaled.view(B, T, H, Nh).copy_(qv)
                    qsrc = ws.qscaled
                # the carried state enters through the epilogue (decayed by gamma^T per
                # head), and the bf16 operand copy for the next chunk leaves with it
                src = rho0s[l] if rho0s is not None else None
                G.gemm(G.EPI_F32, Operand(qsrc, True, Nh, T, N, z1=(H, Nh), z2=(B, T * N)),
                       Operand(v16, True, D, T, D, z2=(B, T * D)), Nh, D, T, ro, Z1=H, Z2=B, ld=D, sz1=Nh * D,
                       sz2=H * Nh * D, accumulate=src is not None, acc_src=src,
                       src_decay_T=T if (decay and src is not None) else 0, log2_decay=ws.log2_decay,
                       out1=out16[l] if out16 is not None else None)
            mod.ln_fwd(ws.a32[l], None, M * H, D, p32["norm_gamma"], p32["norm_beta"], eps, None, ws.an16[l],
                       ws.amean[l], ws.arstd[l], **nk)
            # yn = relu(an Dy - thr) * x                (K = D)
            G.gemm(G.EPI_GATE, Operand(ws.an16[l], False, D, M, H * D, z1=(H, D)), B_encv, M, Nh, D, ws.yn16[l],
                   Z1=H, bn=G.tma_bn(M, Nh), aux0=ws.x16[l], ld=N, sz1=Nh, thr=thr_y)
            # m = yn E (split-K partials), v' = LN(v + LN(m))
            if peer is not None:
                # decoder product with the reduce-scatter fused into its epilogue, then the
                # owners' sums all-gathered by peer stores (parallel.tp.PeerSum)
                G.gemm(G.EPI_F32_SCATTER, Operand(ws.yn16[l], False, N, M, N), B_dec, M, D, N, ws.m32[l], ld=D,
                       scatter=peer.scatter_args())
                if self.tp.sequence_parallel:
                    # the owner merges its own rows and gathers their bf16 copies
                    peer.sp_tail_forward(l, ws.v32[l], ws.v32[l + 1], ws.tst[l], p32["norm_gamma"],
                                         p32["norm_beta"], eps, nk)
                    continue
                peer.finish(l)
                mod.tail_fwd(ws.m32[l], 1, M * D, ws.v32[l], M, D, p32["norm_gamma"], p32["norm_beta"], eps, None,
                             ws.v32[l + 1], ws.v16[l + 1], ws.tst[l], **nk)
                continue
            G.gemm(G.EPI_F32, Operand(ws.yn16[l], False, N, M, N), B_dec, M, D, N, ws.partial,
                   splits=ws.dec_splits, ld=D, split_stride=M * D)
            if self.tp is not None and self.tp.world > 1:
                # sum this rank's split-K partials, then over the tensor-parallel group
                msum = ws.partial[0]
                if ws.dec_splits > 1:
                    mod.sum_rows(ws.m32[l], msum, ws.partial[1:], ws.dec_splits - 1, M * D, None, 0, 0, M * D)
                else:
                    ws.m32[l].copy_(msum)
                self.tp.all_reduce(ws.m32[l])
                mod.tail_fwd(ws.m32[l], 1, M * D, ws.v32[l], M, D, p32["norm_gamma"], p32["norm_beta"], eps, None,
                             ws.v32[l + 1], ws.v16[l + 1], ws.tst[l], **nk)
            else:
                mod.tail_fwd(ws.partial, ws.dec_splits, M * D, ws.v32[l], M, D, p32["norm_gamma"],
                             p32["norm_beta"], eps, ws.m32[l], ws.v32[l + 1], ws.v16[l + 1], ws.tst[l], **nk)
        if with_head:
            G.gemm(G.EPI_F32, Operand(ws.v16[L], False, D, M, D), Operand(p16["lm_head"], True, ws.V, D, ws.V),
                   M, ws.V, D, ws.logits, ld=ws.V)
        return out_states

    def loss(self, targets: torch.Tensor, mask: torch.Tensor | None = None, scale: float = 1.0) -> torch.Tensor:
        """Token-mean CE; ``scale`` multiplies the loss and its gradient (1/n for an
        n-micro-batch accumulation)."""
        ws = self.ws
        if mask is not None:
            ws.inv_count.copy_(scale / mask.float().sum().clamp_min(1.0))
            m = mask.reshape(-1).float().contiguous()
        else:
            ws.inv_count.fill_(scale / ws.M)
            m = None
        self.mod.cross_entropy(ws.logits, targets.reshape(-1).contiguous(), m, ws.inv_count, ws.M, ws.V, ws.loss_rows,
                               ws.dlogits16)
        return ws.loss_rows.sum() * ws.inv_count[0]

    # ---------------------------------------------------------------- backward
    def backward(self, p16: dict, p32: dict, g32: dict, tokens: torch.Tensor | None, pos0: int = 0,
                 accumulate: bool = False, dv_out: torch.Tensor | None = None, with_embed: bool = True,
                 grad_ready=None, grad16: dict | None = None):
        """Writes parameter gradients into g32 (``accumulate``: adds to them, for
        gradient accumulation over micro-batches).

        Pipeline stages: ``dv_out`` ([M, D] fp32, the gradient of this stage's output)
        replaces the LM head / CE backward; ``with_embed=False`` stops at this stage's
        input and returns its gradient (a view of a workspace buffer).

        ``grad_ready(name)``: called once layer 0 has added its last term to the shared
        ``decoder`` / ``encoder_v`` / ``encoder`` gradient and the backward has finished
        reading that projection's bf16 shadow (the data-parallel exchange may then
        overwrite it). ``grad16``: bf16 destinations of those gradients; layer 0's weight
        GEMMs write the final values there too (the exchange's transport copy, no
        conversion pass)."""
        ready = grad_ready if grad_ready is not None else (lambda name: None)
        g16 = grad16 or {}
        ws, cfg, mod = self.ws, self.cfg, self.mod
        B, T, D, H, Nh, N, M, L, V = ws.B, ws.T, ws.D, ws.H, ws.Nh, ws.N, ws.M, ws.L, ws.V
        gam, bet = p32["norm_gamma"], p32["norm_beta"]
        nk = norm_kwargs(cfg, p32)
        tp = self.tp if self.tp is not None and self.tp.world > 1 else None
        if not accumulate:
            for k in ("encoder", "encoder_v", "decoder"):
                g32[k].zero_()
        parts = []       # norm-grad partials identical on every tensor-parallel rank
        head_parts = []  # norm-grad partials of this rank's heads (summed over the group)
        dv = ws.dv[0]
        if dv_out is None:
            # lm head
            G.gemm(G.EPI_F32, Operand(ws.v16[L], True, D, M, D), Operand(ws.dlogits16, True, V, M, V), D, V, M,
                   g32["lm_head"], ld=V, accumulate=accumulate)
            G.gemm(G.EPI_F32, Operand(ws.dlogits16, False, V, M, V), Operand(p16["lm_head"], False, V, D, V), M, D,
                   V, dv, ld=D)
        else:
            if not accumulate and "lm_head" in g32:
                g32["lm_head"].zero_()
            dv.copy_(dv_out.reshape(M, D))
        enc, encv, dec = p16["encoder"], p16["encoder_v"], p16["decoder"]
        sp = tp is not None and tp.sequence_parallel and tp.peer is not None
        own = tp.peer.own_rows() if sp else None
        for l in reversed(range(L)):
            v16 = ws.v16[l]
            if sp:
                # residual-merge backward on this rank's rows; the bf16 decoder gradient rows
                # are gathered, the LayerNorm partials summed over the group below
                rows = own.stop - own.start
                head_parts.append(mod.tail_bwd(dv[own], ws.v32[l][own], tp.peer.m_own[l], ws.tst[l][own], rows, D,
                                               gam, bet, ws.dm16[own], ws.dv_res[own], **nk))
                tp.peer.sp_gather_dm()
            else:
                parts.append(mod.tail_bwd(dv, ws.v32[l], ws.m32[l], ws.tst[l], M, D, gam, bet, ws.dm16, ws.dv_res, **nk))
            # d(yn) = dm E^T -> dx_part = d(yn)*y, dy_pre = d(yn)*x*[y>0]
            G.gemm(G.EPI_DEC_BWD, Operand(ws.dm16, False, D, M, D), Operand(dec, False, D, N, D), M, N, D, ws.dx16, bn=G.tma_bn(M, N),
                   out1=ws.dy16, aux0=ws.x16[l], aux1=ws.yn16[l], ld=N)
            # dE += yn^T dm
            G.gemm(G.EPI_F32, Operand(ws.yn16[l], True, N, M, N), Operand(ws.dm16, True, D, M, D), N, D, M,
                   g32["decoder"], ld=D, accumulate=True, out1=g16.get("decoder") if l == 0 else None)
            if l == 0:
                ready("decoder")
            # dDy_h += an_h^T dy_h
            G.gemm(G.EPI_F32, Operand(ws.an16[l], True, D, M, H * D, z1=(H, D)),
                   Operand(ws.dy16, True, Nh, M, N, z1=(H, Nh)), D, Nh, M, g32["encoder_v"], Z1=H, ld=Nh,
                   sz1=D * Nh, accumulate=True, out1=g16.get("encoder_v") if l == 0 else None)
            # d(an)_h = dy_h Dy_h^T
            G.gemm(G.EPI_F32, Operand(ws.dy16, False, Nh, M, N, z1=(H, Nh)),
                   Operand(encv, False, Nh, D, Nh, z1=(H, D * Nh)), M, D, Nh, ws.dan32, Z1=H, ld=H * D, sz1=D)
            if l == 0:
                # after the last read of the encoder_v shadow: its new weights may land now
                ready("encoder_v")
            # dC = LN^T(d an), written as [B,H,T,D]
            head_parts.append(mod.ln_bwd(ws.dan32, ws.a32[l], ws.amean[l], ws.arstd[l], M * H, D, gam, T, H, ws.dC16,
                                    None, **nk))
            # P = dC V^T ; G = mask(P) + mask(P)^T
            dcop = Operand(ws.dC16, False, D, T, D, z1=(H, T * D), z2=(B, H * T * D))
            G.gemm(G.EPI_F32, dcop, Operand(v16, False, D, T, D, z2=(B, T * D)), T, T, D, ws.P32, Z1=H, Z2=B,
                   bn=128 if T % 128 == 0 else 64, ld=T, sz1=T * T, sz2=H * T * T)
            mod.symmetrize(ws.P32, ws.G16, B * H, T, H, ws.log2_decay)
            # dx_pre = (dx_part + rope^T(G q)) * [x > 0]   (in place over dx_part, which
            # carries the x <= 0 mask as -0.0 from the decoder backward)
            G.gemm(G.EPI_DQ, Operand(ws.G16, False, T, T, T, z1=(H, T * T), z2=(B, H * T * T)),
                   Operand(ws.q16[l], True, Nh, T, N, z1=(H, Nh), z2=(B, T * N)), T, Nh, T, ws.dx16, Z1=H, Z2=B,
                   bn=G.tma_bn(T, Nh, "dq"),
                   aux0=ws.dx16, ld=N, sz1=Nh, sz2=T * N, freq=ws.freq, pos0=pos0, T=T, Nh=Nh,
                   rope_tab=ws.rope_tab(pos0))
            if ws.has_rho0:
                # + rope^T(gamma^t dC rho0^T) (the carried state is detached: no grad to rho0)
                G.gemm(G.EPI_DQ, dcop, Operand(ws.rho16[l], False, D, Nh, D, z1=(H, Nh * D), z2=(B, H * Nh * D)),
                       T, Nh, D, ws.dx16, Z1=H, Z2=B, bn=128, aux0=ws.dx16, ld=N, sz1=Nh,
                       sz2=T * N, freq=ws.freq, pos0=pos0, T=T, Nh=Nh, log2_decay=ws.log2_decay,
                       rope_tab=ws.rope_tab(pos0),
                       row_decay=ws.log2_decay is not None)
            # dV = sum_h S_h^T dC_h  (K = (h, i))
            G.gemm(G.EPI_F32, Operand(ws.S16[l], True, T, H * T, T, z2=(B, H * T * T)),
                   Operand(ws.dC16, True, D, H * T, D, z2=(B, H * T * D)), T, D, H * T, ws.dva32, Z2=B, ld=D,
                   sz2=T * D)
            # dDx_h += v^T dx_h
            G.gemm(G.EPI_F32, Operand(v16, True, D, M, D), Operand(ws.dx16, True, Nh, M, N, z1=(H, Nh)), D, Nh, M,
                   g32["encoder"], Z1=H, ld=Nh, sz1=D * Nh, accumulate=True,
                   out1=g16.get("encoder") if l == 0 else None)
            # dv_x per head = dx_h Dx_h^T
            G.gemm(G.EPI_F32, Operand(ws.dx16, False, Nh, M, N, z1=(H, Nh)),
                   Operand(enc, False, Nh, D, Nh, z1=(H, D * Nh)), M, D, Nh, ws.dvx32, Z1=H, ld=D, sz1=M * D)
            if l == 0:
                # after the last read of the encoder shadow
                ready("encoder")
            dv_next = ws.dv[1] if dv is ws.dv[0] else ws.dv[0]
            if sp:
                # reduce-scatter only: the owner's rows get the group sum plus its residual
                mod.sum_rows(dv_next, None, ws.dvx32, H, M * D, ws.dva32, 1, 0, M * D)
                tp.peer.sp_reduce_scatter(dv_next, ws.dv_res[own])
            elif tp is not None:
                mod.sum_rows(dv_next, None, ws.dvx32, H, M * D, ws.dva32, 1, 0, M * D)
                if tp.peer is not None and tp.peer.M == M and tp.peer.D == D:
                    tp.peer.all_reduce_rows(dv_next)  # P2P scatter / owner sum / P2P gather
                else:
                    tp.all_reduce(dv_next)
                dv_next.add_(ws.dv_res)
            else:
                mod.sum_rows(dv_next, ws.dv_res, ws.dvx32, H, M * D, ws.dva32, 1, 0, M * D)
            dv = dv_next
        if with_embed:
            # embedding LayerNorm and gather
            demb = ws.dv_res  # reuse as fp32 [M, D] scratch
            if sp:
                rows = own.stop - own.start
                tok = ws.token_ids(tokens)[own]
                head_parts.append(mod.ln_bwd(dv[own], p32["embed"], ws.emean[own], ws.erstd[own], rows, D, gam,
                                             0, 0, None, demb[own], **nk, tokens=tok))
                ge = torch.empty_like(g32["embed"])
                embed_grad(mod, tokens.reshape(-1)[own].contiguous(), demb[own], ge, accumulate=False)
                tp.all_reduce(ge)  # every rank's own-row contributions
                if accumulate:
                    g32["embed"].add_(ge)
                else:
                    g32["embed"].copy_(ge)
            else:
                parts.append(mod.ln_bwd(dv, p32["embed"], ws.emean, ws.erstd, M, D, gam, 0, 0, None, demb, **nk,
                                        tokens=ws.token_ids(tokens)))
                embed_grad(mod, tokens.reshape(-1), demb, g32["embed"], accumulate=accumulate)
        elif not accumulate:
            g32["embed"].zero_()
        allp = torch.cat(parts, 0).sum(0) if parts else 0.0
        hp = torch.cat(head_parts, 0).sum(0)
        if tp is not None:
            tp.all_reduce(hp)
        allp = allp + hp
        # rows: dgamma, dbeta (and per-column dalpha / dshift partials for the elementwise kinds)
        grads = [("norm_gamma", allp[0]), ("norm_beta", allp[1])]
        if nk["norm_kind"] >= 2:
            grads += [("norm_alpha", allp[2].sum().reshape(1)), ("norm_shift", allp[3].sum().reshape(1))]
        elif "norm_alpha" in g32 and not accumulate:
            g32["norm_alpha"].zero_()
            g32["norm_shift"].zero_()
        for name, gv in grads:
            if accumulate:
                g32[name].add_(gv)
            else:
                g32[name].copy_(gv)
        return None if with_embed else dv
