"""Mamba language model whose selective scans run on the CUDA op.

The reference project ships only the scan op; a Mamba graph around it is the
caller's (its block dataflow is benchmarks/profiler.py:18-150: in_proj ->
causal depthwise conv1d + SiLU -> x_proj -> dt_proj + softplus -> scan ->
x SiLU(z) -> out_proj). This module is that caller, written in torch for the
GEMMs, the convolution and the norms, with every scan sent through
``mamba_onnx.cuda.selective_scan`` as ``SelectiveScanFusedExact`` (abar =
exp(delta*A), softplus(delta + dt_proj.bias) fused into the op through its
``delta_bias`` input). Parameter names and shapes follow transformers'
``MambaForCausalLM`` so its weights load directly; its ``MambaMixer.slow_forward``
is the numerical reference.

Everything is float32. On CUDA the large projections (in_proj, out_proj and
the LM head) over 16 or more tokens run on this package's tensor-core GEMM in
3xTF32 form (operands split into two tf32 parts, three products summed with
fp32 accumulation: fp32-accurate; ``GEMM = "cublas"`` selects torch's fp32
GEMMs instead); single-token steps use torch's fp32 GEMMs for those
projections. x_proj, whose 80-wide output is too narrow to fill the GPU with
GEMM tiles, runs on this package's fp32 kernel (d_inner split over a cluster
of 8 CTAs, or one warp per output when decoding; dt, B and C written apart),
and dt_proj on this package's K = dt_rank kernel, which writes the scan's
[B, D, L] delta (``DT_PROJ`` selects it fused behind x_proj, each CTA of the
cluster forming delta for its own d_inner rows, or torch's fp32 GEMM
instead). ``forward`` runs a whole
sequence; ``step`` decodes one
token from a ``DecodeState`` (the convolution window and the 16 scan states
per channel), which the scan carries in through ``h0`` and out through
``h_last``. On CUDA tensors the RMSNorms and the causal convolution + SiLU run
on this package's kernels too (include/mamba_model_ops.h); on CPU tensors the
same arithmetic runs as torch operations.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import cuda

SCAN_OP = "SelectiveScanFusedExact"
# decoding on CUDA: one persistent kernel per token ("persistent"; batch <= 4,
# d_model <= 1024, d_inner <= 2048, dt_rank <= 64, d_conv <= 4, else the
# chain) or the chain of per-block kernels ("chain"); both give the same values
DECODE = "persistent"
# dt_proj on CUDA: this package's standalone kernel ("kernel"), fused behind
# x_proj ("fused", dt_rank <= 96; else "kernel") or torch's fp32 GEMM ("cublas")
DT_PROJ = "kernel"


@dataclass(frozen=True)
class MambaConfig:
    d_model: int = 768
    n_layer: int = 24
    vocab_size: int = 50280
    d_state: int = 16
    d_conv: int = 4
    expand: int = 2
    dt_rank: int = 0  # 0: ceil(d_model / 16)
    rms_eps: float = 1e-5

    @property
    def d_inner(self) -> int:
        return self.expand * self.d_model

    @property
    def rank(self) -> int:
        return self.dt_rank or math.ceil(self.d_model / 16)


def rms_norm(x, weight, eps: float):
    """x * rsqrt(mean(x^2, -1) + eps) * weight (one CUDA kernel on CUDA tensors)."""
    if x.is_cuda:
        return cuda.rmsnorm(x.contiguous(), weight, eps)
    var = x.pow(2).mean(-1, keepdim=True)
    return x * torch.rsqrt(var + eps) * weight


def conv_silu(x, weight, bias):
    """silu(causal depthwise conv1d over the last axis): x [B, D, L] (rows
    contiguous, e.g. the first half of the in_proj output), weight [D, 1, K]."""
    if x.is_cuda:
        return cuda.causal_conv1d_silu(x, weight, bias)
    K, L = weight.shape[-1], x.shape[-1]
    return F.silu(F.conv1d(x, weight, bias, padding=K - 1, groups=x.shape[1])[..., :L])


# Dense projections of at least this many tokens run on the tensor-core
# 3xTF32 GEMM (cuda.gemm_tf32x3, fp32-accurate) when GEMM == "tf32x3"; fewer
# tokens (decoding) and GEMM == "cublas" use torch's fp32 GEMMs (TF32 off).
GEMM = "tf32x3"
TC_MIN_TOKENS = 16


def _use_tc(x, tokens: int) -> bool:
    return x.is_cuda and GEMM == "tf32x3" and tokens >= TC_MIN_TOKENS


class _SplitWeight:
    """A weight's tf32 split (cuda.split_tf32), redone when the weight changes."""

    def __init__(self):
        self.key, self.split = None, None

    def get(self, w):
        key = (w.data_ptr(), w._version, tuple(w.shape))
        if self.key != key:
            self.split, self.key = cuda.split_tf32(w.detach()), key
        return self.split


_gemm_workspaces = {}


def _gemm_workspace(device, nbytes: int):
    """The tensor-core GEMM's split-K workspace (cuda.gemm_workspace_size) for
    the current stream of ``device``: one buffer per device and stream, so
    that the calls sharing it are ordered; grown on demand. None for 0 bytes."""
    if nbytes == 0:
        return None
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    ws = _gemm_workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(nbytes, dtype=torch.uint8, device=device)
        _gemm_workspaces[key] = ws
    return ws


def add_out_proj(h, y, weight, split=None):
    """h + y^T W^T for h [B, L, d], y [B, D, L]; the sum is the GEMM's own
    accumulation (addmm, or the tensor-core GEMM's c_in), not a separate kernel.
    A short sequence (few output tiles for a K of d_inner) splits K across the
    SMs through a workspace."""
    if split is not None and _use_tc(h, h.shape[1]):
        w = split.get(weight)
        out = torch.empty_like(h)
        ws = _gemm_workspace(h.device, cuda.gemm_workspace_size(w.rows, h.shape[1], w.cols))
        for b in range(h.shape[0]):  # out[b] [L, d] = h[b] + (y[b]^T [L, D]) W^T
            cuda.gemm_tf32x3(w, cuda.split_tf32(y[b], transpose=True), out[b],
                             transpose_c=True, c_in=h[b], workspace=ws)
        return out
    if h.shape[0] == 1:
        return torch.addmm(h[0], y[0].t(), weight.t()).unsqueeze(0)
    return h + torch.matmul(y.transpose(1, 2), weight.t())


def mamba_130m() -> MambaConfig:
    """Mamba-130m: 24 blocks, d_model 768, d_inner 1536, d_state 16, dt_rank 48."""
    return MambaConfig()


class MambaLayer(torch.nn.Module):
    """One residual block: x + mixer(rmsnorm(x))."""

    def __init__(self, cfg: MambaConfig):
        super().__init__()
        d, D, N, R = cfg.d_model, cfg.d_inner, cfg.d_state, cfg.rank
        f32 = dict(dtype=torch.float32)
        self.cfg = cfg
        self.norm_weight = torch.nn.Parameter(torch.ones(d, **f32))
        self.in_proj_weight = torch.nn.Parameter(torch.empty(2 * D, d, **f32))
        self.conv_weight = torch.nn.Parameter(torch.empty(D, 1, cfg.d_conv, **f32))
        self.conv_bias = torch.nn.Parameter(torch.zeros(D, **f32))
        self.x_proj_weight = torch.nn.Parameter(torch.empty(R + 2 * N, D, **f32))
        self.dt_proj_weight = torch.nn.Parameter(torch.empty(D, R, **f32))
        self.dt_proj_bias = torch.nn.Parameter(torch.empty(D, **f32))
        self.A_log = torch.nn.Parameter(torch.empty(D, N, **f32))
        self.D = torch.nn.Parameter(torch.ones(D, **f32))
        self.out_proj_weight = torch.nn.Parameter(torch.empty(d, D, **f32))
        self._in_split, self._out_split = _SplitWeight(), _SplitWeight()
        self._A_key, self._A = None, None

    def A(self):
        """-exp(A_log), recomputed only when A_log changes."""
        key = (self.A_log.data_ptr(), self.A_log._version, self.A_log.device)
        if self._A_key != key:
            with torch.no_grad():
                self._A, self._A_key = -torch.exp(self.A_log), key
        return self._A

    def _norm(self, x):
        return rms_norm(x, self.norm_weight, self.cfg.rms_eps)

    def _ssm_inputs(self, x):
        """x [B, D, L] after conv + SiLU -> delta [B, D, L] (before bias), B, C [B, L, N]."""
        N, R = self.cfg.d_state, self.cfg.rank
        if x.is_cuda:  # this package's x_proj: dt, B, C written apart, no copies
            if DT_PROJ == "fused" and R <= cuda.X_PROJ_DELTA_MAX_RANK:
                return cuda.x_proj_delta(x.contiguous(), self.x_proj_weight.detach(),
                                         self.dt_proj_weight.detach(), R, N)
            dt, Bm, Cm = cuda.x_proj(x.contiguous(), self.x_proj_weight.detach(), R, N)
            if DT_PROJ == "cublas":
                if x.shape[0] == 1:  # a 2-D GEMM on the transposed view writes [D, L] directly
                    return torch.mm(self.dt_proj_weight, dt[0].t()).unsqueeze(0), Bm, Cm
                return torch.matmul(self.dt_proj_weight, dt.transpose(1, 2)), Bm, Cm
            return cuda.dt_proj(dt, self.dt_proj_weight.detach()), Bm, Cm  # [B, D, L]
        if x.shape[0] == 1:  # 2-D GEMMs take the transposed views without copies
            x_dbl = torch.mm(x[0].t(), self.x_proj_weight.t()).unsqueeze(0)  # [1, L, R + 2N]
            delta = torch.mm(self.dt_proj_weight, x_dbl[0, :, :R].t()).unsqueeze(0)
        else:
            x_dbl = torch.matmul(x.transpose(1, 2), self.x_proj_weight.t())  # [B, L, R + 2N]
            delta = torch.matmul(self.dt_proj_weight, x_dbl[..., :R].transpose(1, 2))  # [B, D, L]
        Bm = x_dbl[..., R:R + N].contiguous()
        Cm = x_dbl[..., R + N:].contiguous()
        return delta, Bm, Cm

    def _in_proj(self, h):
        """rmsnorm(h) [B, L, d] -> in_proj output xz [B, 2D, L] (x rows, then z rows)."""
        if _use_tc(h, h.shape[1]) and h.shape[-1] % 4 == 0:
            # the norm writes the GEMM operand's tf32 parts directly
            hs = cuda.rmsnorm_split_tf32(h.contiguous(), self.norm_weight.detach(),
                                         self.cfg.rms_eps)
            w = self._in_split.get(self.in_proj_weight)
            L = h.shape[1]
            xz = torch.empty(h.shape[0], w.rows, L, device=h.device)
            for b in range(h.shape[0]):  # xz[b] [2D, L] = W hn[b]^T
                cuda.gemm_tf32x3(w, hs.row_block(b * L, L), xz[b])
            return xz
        hn = self._norm(h)
        if _use_tc(h, h.shape[1]):
            w = self._in_split.get(self.in_proj_weight)
            xz = torch.empty(h.shape[0], w.rows, h.shape[1], device=h.device)
            for b in range(h.shape[0]):
                cuda.gemm_tf32x3(w, cuda.split_tf32(hn[b]), xz[b])
            return xz
        if h.shape[0] == 1:
            return torch.mm(self.in_proj_weight, hn[0].t()).unsqueeze(0)
        return torch.matmul(self.in_proj_weight, hn.transpose(1, 2))

    def forward(self, h, A, conv_state=None, ssm_state=None, scan=None):
        """h [B, L, d_model] -> h + mixer(norm(h)); A = -exp(A_log). Given
        conv_state [B, D, d_conv] and ssm_state [B, D, N], they receive the
        state after the last token (for decoding on from here). ``scan``
        replaces the CUDA op (same signature as cuda.selective_scan)."""
        scan = scan or cuda.selective_scan
        D, L, K = self.cfg.d_inner, h.shape[1], self.cfg.d_conv
        xz = self._in_proj(h)  # [B, 2D, L]
        x = conv_silu(xz[:, :D], self.conv_weight, self.conv_bias)
        z = xz[:, D:].contiguous()
        delta, Bm, Cm = self._ssm_inputs(x)
        y = scan(SCAN_OP, x, delta, A, Bm, Cm, self.D, z, delta_bias=self.dt_proj_bias,
                 h_last=ssm_state)
        if conv_state is not None:  # the last K inputs of the convolution, zero-padded
            conv_state.copy_(F.pad(xz[:, :D], (max(0, K - L), 0))[..., -K:])
        return add_out_proj(h, y, self.out_proj_weight, self._out_split)

    def step(self, h, A, conv_state, ssm_state):
        """One token: h [B, 1, d_model]; conv_state [B, D, d_conv] (last inputs of
        the convolution, oldest first) and ssm_state [B, D, N] are updated."""
        D, N, R = self.cfg.d_inner, self.cfg.d_state, self.cfg.rank
        if h.is_cuda:
            # this package's kernels: RMSNorm + in_proj, the convolution step
            # (window shift, conv, SiLU), x_proj, dt_proj + the scan step + the
            # state update in one kernel (SelectiveScanFusedExact at seqlen 1),
            # then out_proj + the residual
            xz = cuda.rmsnorm_gemv(h[:, 0], self.norm_weight.detach(), self.cfg.rms_eps,
                                   self.in_proj_weight.detach()).unsqueeze(-1)  # [B, 2D, 1]
            x = cuda.causal_conv1d_step(conv_state, xz[:, :D, 0], self.conv_weight.detach(),
                                        self.conv_bias.detach())  # [B, D]
            dt, Bm, Cm = cuda.x_proj(x.unsqueeze(-1), self.x_proj_weight.detach(), R, N)
            y = cuda.ssm_decode_step(x, xz[:, D:, 0], dt[:, 0], Bm[:, 0], Cm[:, 0],
                                     self.dt_proj_weight.detach(), self.dt_proj_bias.detach(),
                                     A, self.D.detach(), ssm_state)
            return cuda.gemv(y, self.out_proj_weight.detach(), residual=h[:, 0]).unsqueeze(1)
        # the same step in torch operations around the scan op
        xz = self._in_proj(h)  # [B, 2D, 1]
        conv_state.copy_(torch.cat([conv_state[..., 1:], xz[:, :D]], dim=-1))
        x = torch.sum(conv_state * self.conv_weight[:, 0, :], dim=-1) + self.conv_bias
        x = F.silu(x).unsqueeze(-1).contiguous()  # [B, D, 1]
        z = xz[:, D:].contiguous()
        delta, Bm, Cm = self._ssm_inputs(x)
        new_state = torch.empty_like(ssm_state)
        y = cuda.selective_scan(SCAN_OP, x, delta, A, Bm, Cm, self.D, z,
                                delta_bias=self.dt_proj_bias, h0=ssm_state, h_last=new_state)
        ssm_state.copy_(new_state)
        return add_out_proj(h, y, self.out_proj_weight)


@dataclass
class DecodeState:
    conv: list  # per layer [B, D, d_conv]
    ssm: list   # per layer [B, D, N]


class MambaLM(torch.nn.Module):
    """Embedding -> n_layer MambaLayers -> RMSNorm -> tied LM head."""

    def __init__(self, cfg: MambaConfig):
        super().__init__()
        self.cfg = cfg
        self.embedding = torch.nn.Parameter(torch.empty(cfg.vocab_size, cfg.d_model))
        self.layers = torch.nn.ModuleList(MambaLayer(cfg) for _ in range(cfg.n_layer))
        self.norm_f_weight = torch.nn.Parameter(torch.ones(cfg.d_model))
        self._emb_split = _SplitWeight()

    # ---------------------------------------------------------------- weights

    @torch.no_grad()
    def init_random(self, seed: int = 0, dt_min: float = 1e-3, dt_max: float = 1e-1):
        """Mamba's initialisation: A_log = log(1..N) per channel (S4D-real),
        dt log-uniform in [dt_min, dt_max] with dt_proj.bias = softplus^-1(dt),
        D = 1, conv and projections N(0, 0.02) (conv bias 0)."""
        g = torch.Generator(device="cpu").manual_seed(seed)
        cfg = self.cfg
        normal = lambda t: t.copy_(torch.randn(t.shape, generator=g) * 0.02)  # noqa: E731
        normal(self.embedding)
        for layer in self.layers:
            for w in (layer.in_proj_weight, layer.conv_weight, layer.x_proj_weight,
                      layer.dt_proj_weight, layer.out_proj_weight):
                normal(w)
            layer.conv_bias.zero_()
            layer.norm_weight.fill_(1.0)
            dt = torch.exp(torch.rand(cfg.d_inner, generator=g)
                           * (math.log(dt_max) - math.log(dt_min)) + math.log(dt_min))
            layer.dt_proj_bias.copy_(dt + torch.log(-torch.expm1(-dt)))
            layer.A_log.copy_(torch.log(torch.arange(1, cfg.d_state + 1, dtype=torch.float32))
                              .repeat(cfg.d_inner, 1))
            layer.D.fill_(1.0)
        self.norm_f_weight.fill_(1.0)
        return self

    HF_NAMES = {
        "norm_weight": "norm.weight",
        "in_proj_weight": "mixer.in_proj.weight",
        "conv_weight": "mixer.conv1d.weight",
        "conv_bias": "mixer.conv1d.bias",
        "x_proj_weight": "mixer.x_proj.weight",
        "dt_proj_weight": "mixer.dt_proj.weight",
        "dt_proj_bias": "mixer.dt_proj.bias",
        "A_log": "mixer.A_log",
        "D": "mixer.D",
        "out_proj_weight": "mixer.out_proj.weight",
    }

    @torch.no_grad()
    def load_hf_state_dict(self, sd: dict):
        """Copy weights from a transformers MambaForCausalLM state dict."""
        self.embedding.copy_(sd["backbone.embeddings.weight"])
        self.norm_f_weight.copy_(sd["backbone.norm_f.weight"])
        for i, layer in enumerate(self.layers):
            for ours, theirs in self.HF_NAMES.items():
                getattr(layer, ours).copy_(sd[f"backbone.layers.{i}.{theirs}"])
        return self

    # ---------------------------------------------------------------- forward

    def _head(self, h):
        if _use_tc(h, h.shape[1]) and h.shape[-1] % 4 == 0:
            hs = cuda.rmsnorm_split_tf32(h.contiguous(), self.norm_f_weight.detach(),
                                         self.cfg.rms_eps)
            e = self._emb_split.get(self.embedding)
            L = h.shape[1]
            logits = torch.empty(h.shape[0], L, e.rows, device=h.device)
            for b in range(h.shape[0]):  # logits[b] [L, V] = hn[b] E^T
                cuda.gemm_tf32x3(hs.row_block(b * L, L), e, logits[b])
            return logits
        h = rms_norm(h, self.norm_f_weight, self.cfg.rms_eps)
        if _use_tc(h, h.shape[1]):
            e = self._emb_split.get(self.embedding)
            logits = torch.empty(h.shape[0], h.shape[1], e.rows, device=h.device)
            for b in range(h.shape[0]):  # logits[b] [L, V] = h[b] E^T
                cuda.gemm_tf32x3(cuda.split_tf32(h[b]), e, logits[b])
            return logits
        return torch.matmul(h, self.embedding.t())

    @torch.no_grad()
    def forward(self, input_ids, scan=None):
        """input_ids [B, L] int64 -> logits [B, L, vocab]. ``scan`` replaces the
        CUDA op in every layer (same signature as cuda.selective_scan); by
        default the scans run on cuda.selective_scan and need a CUDA device."""
        h = F.embedding(input_ids, self.embedding)
        for layer in self.layers:
            h = layer(h, layer.A(), scan=scan)
        return self._head(h)

    @torch.no_grad()
    def prefill(self, input_ids):
        """forward() that also returns the DecodeState after the last token."""
        state = self.new_state(input_ids.shape[0])
        h = F.embedding(input_ids, self.embedding)
        for layer, cs, ss in zip(self.layers, state.conv, state.ssm):
            h = layer(h, layer.A(), cs, ss)
        return self._head(h), state

    def new_state(self, batch: int) -> DecodeState:
        cfg, dev = self.cfg, self.embedding.device
        return DecodeState(
            conv=[torch.zeros(batch, cfg.d_inner, cfg.d_conv, device=dev) for _ in self.layers],
            ssm=[torch.zeros(batch, cfg.d_inner, cfg.d_state, device=dev) for _ in self.layers])

    def _decode_setup(self, state: DecodeState, batch: int):
        """(table, scratch) of mamba_decode_step for this state, built once per
        state and weight version (the table holds the tensors' addresses)."""
        key = (batch, tuple(t.data_ptr() for t in state.conv + state.ssm),
               tuple((p.data_ptr(), p._version) for p in self.parameters()))
        cached = getattr(self, "_decode_cache", None)
        if cached is None or cached[0] != key:
            cfg = self.cfg
            rows = []
            for layer, cs, ss in zip(self.layers, state.conv, state.ssm):
                rows.append({
                    "norm_weight": layer.norm_weight.detach(),
                    "in_proj_weight": layer.in_proj_weight.detach(),
                    "conv_weight": layer.conv_weight.detach(),
                    "conv_bias": layer.conv_bias.detach(),
                    "x_proj_weight": layer.x_proj_weight.detach(),
                    "dt_proj_weight": layer.dt_proj_weight.detach(),
                    "dt_proj_bias": layer.dt_proj_bias.detach(),
                    "A": layer.A(), "D": layer.D.detach(),
                    "out_proj_weight": layer.out_proj_weight.detach(),
                    "conv_state": cs, "ssm_state": ss})
            table = cuda.decode_layer_table(rows, self.embedding.device)
            scratch = torch.empty(cuda.decode_scratch_size(batch, cfg.d_inner, cfg.rank,
                                                           cfg.d_state),
                                  dtype=torch.uint8, device=self.embedding.device)
            self._decode_cache = (key, table, scratch, [r["A"] for r in rows])
        return self._decode_cache[1], self._decode_cache[2]

    @torch.no_grad()
    def step(self, input_ids, state: DecodeState):
        """One decoding step: input_ids [B] -> logits [B, vocab]; state updated."""
        cfg = self.cfg
        if (input_ids.is_cuda and DECODE == "persistent" and input_ids.shape[0] <= 4
                and cfg.d_model <= 1024 and cfg.d_inner <= 2048 and cfg.rank <= 64
                and cfg.d_conv <= 4 and cfg.d_state == 16):
            table, scratch = self._decode_setup(state, input_ids.shape[0])
            h = F.embedding(input_ids, self.embedding)  # [B, d_model], becomes the last h
            logits = torch.empty(input_ids.shape[0], cfg.vocab_size, device=h.device)
            return cuda.decode_step(table, cfg.n_layer, h, self.norm_f_weight.detach(),
                                    self.embedding.detach(), logits, scratch,
                                    d_inner=cfg.d_inner, d_conv=cfg.d_conv, rank=cfg.rank,
                                    dstate=cfg.d_state, eps=cfg.rms_eps)
        h = F.embedding(input_ids[:, None], self.embedding)
        for layer, cs, ss in zip(self.layers, state.conv, state.ssm):
            h = layer.step(h, layer.A(), cs, ss)
        if h.is_cuda:  # final RMSNorm and the tied LM head in one kernel
            return cuda.rmsnorm_gemv(h[:, 0], self.norm_f_weight.detach(), self.cfg.rms_eps,
                                     self.embedding.detach())
        return self._head(h)[:, 0]

    @torch.no_grad()
    def capture_step(self, batch: int, warmup: int = 3):
        """CUDA-graph one decoding step. Returns (ids, logits, state, graph):
        load a DecodeState into ``state`` (``copy_state``; e.g. from
        ``prefill``), write the next token ids into ``ids``, ``graph.replay()``,
        read ``logits``; ``state`` advances by one token per replay."""
        dev = self.embedding.device
        ids = torch.zeros(batch, dtype=torch.int64, device=dev)
        state = self.new_state(batch)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.step(ids, state)
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            logits = self.step(ids, state)
        for t in state.conv + state.ssm:
            t.zero_()
        return ids, logits, state, graph

    @staticmethod
    @torch.no_grad()
    def copy_state(dst: DecodeState, src: DecodeState):
        for a, b in zip(dst.conv + dst.ssm, src.conv + src.ssm):
            a.copy_(b)

    @torch.no_grad()
    def capture(self, batch: int, seqlen: int, warmup: int = 3):
        """CUDA-graph the forward for a fixed shape. Returns (ids, logits, graph):
        write token ids into ``ids``, ``graph.replay()``, read ``logits``."""
        dev = self.embedding.device
        ids = torch.zeros(batch, seqlen, dtype=torch.int64, device=dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.forward(ids)
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            logits = self.forward(ids)
        return ids, logits, graph
