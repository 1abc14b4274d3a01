"""torch.fx pass that swaps attention subgraphs for the block-sparse kernel.

Drop-in for the upstream ``fx_compiler_pass.py`` (same public names,
configuration, matching rules, installed-module names and errors), so a
model rewritten by it calls :func:`sparse_triton_kernel.block_sparse_attention`
-- here the sm_100a CUDA kernels of ``libsbfa.so``.

Two subgraph shapes are recognised (upstream ``:372-457``, ``:512-548``):

1. the eager motif ``softmax(matmul(q, k.transpose(..)) (*|/) s, dim=-1) @ v``
   (the scale step is optional; ``s`` may be a literal or a module attribute);
2. ``F.scaled_dot_product_attention(q, k, v, ..., is_causal=True)`` with
   zero dropout and a static (or absent) ``scale``.

Each match becomes one ``call_module`` to an :class:`_InjectedTritonAttention`
child named ``_triton_attn_<i>`` (eager matches numbered first), which owns
the shared block mask as a non-persistent buffer.
"""

from __future__ import annotations

import math
import operator
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.fx as fx
import torch.nn as nn
import torch.nn.functional as F  # noqa: N812

from sparse_triton_kernel import StreamingMaskSpec, block_sparse_attention, make_streaming_mask

# ---------------------------------------------------------------------------
# Example eager modules (inputs the pass is written to rewrite)
# ---------------------------------------------------------------------------


class StandardAttention(nn.Module):
    """``softmax(q @ k^T * 1/sqrt(d)) @ v`` written in eager torch
    (upstream ``:54-83``)."""

    def __init__(self, head_dim: int) -> None:
        super().__init__()
        if head_dim <= 0:
            raise ValueError("head_dim must be positive")
        self.head_dim = head_dim
        self.inv_sqrt_d = 1.0 / math.sqrt(head_dim)

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        scores = torch.matmul(q, k.transpose(-2, -1)) * self.inv_sqrt_d
        probs = torch.softmax(scores, dim=-1)
        return torch.matmul(probs, v)


class SingleLayerTransformer(nn.Module):
    """q/k/v/out projections around :class:`StandardAttention`
    (upstream ``:86-116``)."""

    def __init__(self, head_dim: int, model_dim: int) -> None:
        super().__init__()
        self.q_proj = nn.Linear(model_dim, model_dim, bias=False)
        self.k_proj = nn.Linear(model_dim, model_dim, bias=False)
        self.v_proj = nn.Linear(model_dim, model_dim, bias=False)
        self.out_proj = nn.Linear(model_dim, model_dim, bias=False)
        self.attn = StandardAttention(head_dim)
        self.num_heads = model_dim // head_dim
        self.head_dim = head_dim

    def _split(self, x: torch.Tensor) -> torch.Tensor:
        b, n, _ = x.shape
        return x.view(b, n, self.num_heads, self.head_dim).transpose(1, 2)

    def _merge(self, x: torch.Tensor) -> torch.Tensor:
        return x.transpose(1, 2).contiguous().flatten(-2)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        o = self.attn(self._split(self.q_proj(x)), self._split(self.k_proj(x)),
                      self._split(self.v_proj(x)))
        return self.out_proj(self._merge(o))


class _RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6, **kw) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim, **kw))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return y.to(x.dtype) * self.weight


def _rope_rows(table: torch.Tensor, n: int, dtype: torch.dtype) -> torch.Tensor:
    """First ``n`` rows of a RoPE cos/sin table (a leaf of the traced graph)."""
    return table[:n].to(dtype)


fx.wrap("_rope_rows")


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


class _LlamaAttention(nn.Module):
    def __init__(self, hidden: int, n_heads: int, n_kv_heads: int, max_seq: int, theta: float,
                 **kw) -> None:
        super().__init__()
        self.n_heads, self.n_kv_heads, self.head_dim = n_heads, n_kv_heads, hidden // n_heads
        self.q_proj = nn.Linear(hidden, hidden, bias=False, **kw)
        self.k_proj = nn.Linear(hidden, n_kv_heads * self.head_dim, bias=False, **kw)
        self.v_proj = nn.Linear(hidden, n_kv_heads * self.head_dim, bias=False, **kw)
        self.o_proj = nn.Linear(hidden, hidden, bias=False, **kw)
        dev = kw.get("device")
        inv = 1.0 / theta ** (torch.arange(0, self.head_dim, 2, device=dev).float() / self.head_dim)
        ang = torch.outer(torch.arange(max_seq, device=dev).float(), inv)
        ang = torch.cat((ang, ang), dim=-1)
        self.register_buffer("cos", ang.cos(), persistent=False)
        self.register_buffer("sin", ang.sin(), persistent=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        b, n, _ = x.shape
        q = self.q_proj(x).view(b, n, self.n_heads, self.head_dim).transpose(1, 2)
        k = self.k_proj(x).view(b, n, self.n_kv_heads, self.head_dim).transpose(1, 2)
        v = self.v_proj(x).view(b, n, self.n_kv_heads, self.head_dim).transpose(1, 2)
        cos = _rope_rows(self.cos, n, q.dtype)
        sin = _rope_rows(self.sin, n, q.dtype)
        q = q * cos + _rotate_half(q) * sin
        k = k * cos + _rotate_half(k) * sin
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True,
                                           enable_gqa=self.n_kv_heads != self.n_heads)
        return self.o_proj(o.transpose(1, 2).reshape(b, n, self.n_heads * self.head_dim))


class _LlamaBlock(nn.Module):
    def __init__(self, hidden: int, n_heads: int, n_kv_heads: int, mlp: int, max_seq: int,
                 theta: float, **kw) -> None:
        super().__init__()
        self.attn_norm = _RMSNorm(hidden, **kw)
        self.attn = _LlamaAttention(hidden, n_heads, n_kv_heads, max_seq, theta, **kw)
        self.mlp_norm = _RMSNorm(hidden, **kw)
        self.gate = nn.Linear(hidden, mlp, bias=False, **kw)
        self.up = nn.Linear(hidden, mlp, bias=False, **kw)
        self.down = nn.Linear(mlp, hidden, bias=False, **kw)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = x + self.attn(self.attn_norm(x))
        h = self.mlp_norm(x)
        return x + self.down(F.silu(self.gate(h)) * self.up(h))


class LlamaStyleDecoder(nn.Module):
    """Llama-style decoder (RMSNorm, RoPE, SwiGLU MLP, untied LM head) whose
    attention is ``F.scaled_dot_product_attention(..., is_causal=True)`` on
    ``[B, H, N, D]`` transposed views -- the SDPA shape the pass rewrites.
    ``n_kv_heads`` < ``n_heads`` gives grouped-query attention
    (``enable_gqa=True``).  ``forward(ids) -> logits``.  Keyword arguments
    ``device`` / ``dtype`` place and type every parameter at construction."""

    def __init__(self, vocab: int = 32000, hidden: int = 4096, n_layers: int = 8,
                 n_heads: int = 32, mlp: int = 11008, max_seq: int = 32768,
                 rope_theta: float = 10000.0, n_kv_heads: Optional[int] = None, device=None,
                 dtype=None) -> None:
        super().__init__()
        kw = {"device": device, "dtype": dtype}
        n_kv = n_heads if n_kv_heads is None else n_kv_heads
        self.embed = nn.Embedding(vocab, hidden, **kw)
        self.layers = nn.ModuleList(
            _LlamaBlock(hidden, n_heads, n_kv, mlp, max_seq, rope_theta, **kw)
            for _ in range(n_layers))
        self.norm = _RMSNorm(hidden, **kw)
        self.lm_head = nn.Linear(hidden, vocab, bias=False, **kw)

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        x = self.embed(ids)
        for layer in self.layers:
            x = layer(x)
        return self.lm_head(self.norm(x))


# ---------------------------------------------------------------------------
# The installed module
# ---------------------------------------------------------------------------


class _InjectedTritonAttention(nn.Module):
    """Module the pass installs; forwards to :func:`block_sparse_attention`.

    The class name and attributes (``block_mask`` buffer, ``softmax_scale``,
    ``block_m``, ``block_n``, ``is_causal``, ``sink_size``, ``window_size``)
    match upstream ``:124-163`` so code inspecting rewritten graphs keeps
    working.  The mask buffer is non-persistent and follows ``.to(device)``.
    """

    def __init__(self, block_mask: torch.Tensor, softmax_scale: float, block_m: int,
                 block_n: int, is_causal: bool = False, sink_size: int = 0,
                 window_size: int = 0) -> None:
        super().__init__()
        self.register_buffer("block_mask", block_mask, persistent=False)
        self.softmax_scale = float(softmax_scale)
        self.block_m = int(block_m)
        self.block_n = int(block_n)
        self.is_causal = bool(is_causal)
        self.sink_size = int(sink_size)
        self.window_size = int(window_size)

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        return block_sparse_attention(
            q, k, v, self.block_mask, softmax_scale=self.softmax_scale,
            block_m=self.block_m, block_n=self.block_n, is_causal=self.is_causal,
            sink_size=self.sink_size, window_size=self.window_size)


# ---------------------------------------------------------------------------
# Configuration and match records
# ---------------------------------------------------------------------------


@dataclass
class InjectionConfig:
    """What the injected kernel is specialised for (upstream ``:171-203``).

    ``custom_mask`` (a block mask) takes precedence over ``streaming``; one
    of the two is required.  ``head_dim`` only provides the default SDPA
    scale ``1/sqrt(head_dim)``.  The mask is built on the host and moves with
    the rewritten module's ``.to(device)``.
    """

    seq_len_q: int
    seq_len_kv: int
    head_dim: int
    streaming: Optional[StreamingMaskSpec] = None
    custom_mask: Optional[torch.Tensor] = None
    block_m: int = 64
    block_n: int = 64
    device: str | torch.device = "cuda"


@dataclass
class _EagerHit:
    q: fx.Node
    k: fx.Node
    v: fx.Node
    kt: fx.Node            # the transpose of k
    scores: fx.Node        # q @ kt
    scaled: Optional[fx.Node]
    softmax: fx.Node
    out: fx.Node           # probs @ v
    scale: float


@dataclass
class _SdpaHit:
    call: fx.Node
    q: fx.Node
    k: fx.Node
    v: fx.Node
    scale: Optional[float]


_MATMULS = (torch.matmul, operator.matmul)
_SCALERS = (operator.mul, torch.mul, operator.truediv, torch.div)
_DIVIDERS = (operator.truediv, torch.div)
_SOFTMAXES = (torch.softmax, F.softmax)
_SDPA = (F.scaled_dot_product_attention,)


def _fn_call(node: fx.Node, targets) -> bool:
    return node.op == "call_function" and node.target in targets


def _softmax_dim(node: fx.Node):
    if "dim" in node.kwargs:
        return node.kwargs["dim"]
    return node.args[1] if len(node.args) >= 2 else None


def _is_softmax(node: fx.Node) -> bool:
    return _fn_call(node, _SOFTMAXES) or (node.op == "call_method" and node.target == "softmax")


def _is_transpose(node: fx.Node) -> bool:
    if node.op == "call_method":
        return node.target in ("transpose", "mT")
    return node.op == "call_function" and node.target is torch.transpose


def _sdpa_arg(node: fx.Node, name: str, pos: int, default):
    """SDPA argument by keyword or position: (q, k, v, attn_mask, dropout_p,
    is_causal, scale, enable_gqa)."""
    if name in node.kwargs:
        return node.kwargs[name]
    return node.args[pos] if len(node.args) > pos else default


def _static_number(node: fx.Node, owner: nn.Module) -> Optional[float]:
    """The scalar operand of a scale node: a literal, or a module attribute
    holding a number or a one-element tensor; None if not static."""
    for a in node.args:
        if isinstance(a, (int, float)):
            return float(a)
        if isinstance(a, fx.Node) and a.op == "get_attr":
            val = getattr(owner, a.target, None)
            if isinstance(val, (int, float)):
                return float(val)
            if isinstance(val, torch.Tensor) and val.numel() == 1:
                return float(val.item())
            return None
    return None


def _erase_if_dead(graph: fx.Graph, node: fx.Node) -> None:
    if not node.users:
        graph.erase_node(node)


# ---------------------------------------------------------------------------
# The pass
# ---------------------------------------------------------------------------


class BlockSparseAttentionInjector:
    """Trace a module and route its attention through the block-sparse kernel.

    >>> cfg = InjectionConfig(seq_len_q=1024, seq_len_kv=1024, head_dim=64,
    ...                       streaming=StreamingMaskSpec(4, 256))
    >>> fused = BlockSparseAttentionInjector(cfg).transform(model)
    """

    def __init__(self, config: InjectionConfig) -> None:
        self.cfg = config
        self._mask = self._build_mask()

    def _build_mask(self) -> torch.Tensor:
        cfg = self.cfg
        if cfg.custom_mask is not None:
            return cfg.custom_mask.detach().to(device="cpu", dtype=torch.int32).contiguous()
        if cfg.streaming is None:
            raise ValueError("Must supply either `streaming` or `custom_mask`")
        return make_streaming_mask(cfg.seq_len_q, cfg.seq_len_kv, cfg.streaming, cfg.block_m,
                                   cfg.block_n, device="cpu")

    # -- discovery ----------------------------------------------------------

    @staticmethod
    def _eager_hits(graph: fx.Graph, owner: nn.Module) -> List[_EagerHit]:
        hits: List[_EagerHit] = []
        for sm in graph.nodes:
            if not _is_softmax(sm):
                continue
            dim = _softmax_dim(sm)
            if dim is not None and dim != -1:
                continue
            src = sm.args[0] if sm.args else None
            if not isinstance(src, fx.Node):
                continue
            scaled: Optional[fx.Node] = None
            scale = 1.0
            scores = src
            if _fn_call(src, _SCALERS):
                scaled, scores = src, src.args[0]
                num = _static_number(src, owner)
                if num is None:
                    continue
                scale = 1.0 / num if src.target in _DIVIDERS else num
            if not (isinstance(scores, fx.Node) and _fn_call(scores, _MATMULS)):
                continue
            q, kt = scores.args[0], scores.args[1]
            if not (isinstance(q, fx.Node) and isinstance(kt, fx.Node) and _is_transpose(kt)):
                continue
            k = kt.args[0]
            if not isinstance(k, fx.Node):
                continue
            users = list(sm.users)
            if len(users) != 1:
                continue
            out = users[0]
            if not _fn_call(out, _MATMULS) or out.args[0] is not sm:
                continue
            v = out.args[1]
            if not isinstance(v, fx.Node):
                continue
            hits.append(_EagerHit(q, k, v, kt, scores, scaled, sm, out, scale))
        return hits

    @staticmethod
    def _sdpa_hits(graph: fx.Graph) -> List[_SdpaHit]:
        hits: List[_SdpaHit] = []
        for n in graph.nodes:
            if not _fn_call(n, _SDPA) or len(n.args) < 3:
                continue
            q, k, v = n.args[:3]
            if not all(isinstance(t, fx.Node) for t in (q, k, v)):
                continue
            if not bool(_sdpa_arg(n, "is_causal", 5, False)):
                continue  # a non-causal call may carry a dynamic attn_mask
            p = _sdpa_arg(n, "dropout_p", 4, 0.0)
            if isinstance(p, (int, float)) and float(p) != 0.0:
                continue
            s = _sdpa_arg(n, "scale", 6, None)
            if s is not None and not isinstance(s, (int, float)):
                continue
            hits.append(_SdpaHit(n, q, k, v, None if s is None else float(s)))
        return hits

    # -- rewrite ------------------------------------------------------------

    def transform(self, model: nn.Module) -> fx.GraphModule:
        """Return a rewritten ``GraphModule`` (the input model is untouched).

        Raises ``RuntimeError`` when neither pattern occurs.
        """
        gm = fx.symbolic_trace(model)
        eager = self._eager_hits(gm.graph, gm)
        sdpa = self._sdpa_hits(gm.graph)
        if not eager and not sdpa:
            raise RuntimeError(
                "No scaled-dot-product-attention subgraph found (neither the eager "
                "softmax(QKᵀ·s)V motif nor an F.scaled_dot_product_attention(is_causal=True) "
                "call).")
        # names are fixed before rewriting; rewriting runs back to front so a
        # later match still sees the original nodes of an earlier one
        numbered_sdpa = [(len(eager) + i, h) for i, h in enumerate(sdpa)]
        for idx, hit in reversed(numbered_sdpa):
            self._rewrite_sdpa(gm, hit, idx)
        for idx, hit in reversed(list(enumerate(eager))):
            self._rewrite_eager(gm, hit, idx)
        gm.graph.lint()
        gm.recompile()
        return gm

    def _new_module(self, scale: float, causal: bool, sink: int, window: int
                    ) -> _InjectedTritonAttention:
        return _InjectedTritonAttention(block_mask=self._mask, softmax_scale=scale,
                                        block_m=self.cfg.block_m, block_n=self.cfg.block_n,
                                        is_causal=causal, sink_size=sink, window_size=window)

    def _rewrite_sdpa(self, gm: fx.GraphModule, hit: _SdpaHit, idx: int) -> None:
        st = self.cfg.streaming
        scale = hit.scale if hit.scale is not None else 1.0 / math.sqrt(self.cfg.head_dim)
        sink = st.sink_size if st else 0
        window = st.window_size if st else self.cfg.seq_len_kv
        name = f"_triton_attn_{idx}"
        gm.add_submodule(name, self._new_module(scale, True, sink, window))
        with gm.graph.inserting_before(hit.call):
            repl = gm.graph.call_module(name, args=(hit.q, hit.k, hit.v))
        hit.call.replace_all_uses_with(repl)
        _erase_if_dead(gm.graph, hit.call)

    def _rewrite_eager(self, gm: fx.GraphModule, hit: _EagerHit, idx: int) -> None:
        st = self.cfg.streaming
        causal = st is not None
        name = f"_triton_attn_{idx}"
        gm.add_submodule(name, self._new_module(
            hit.scale, causal, st.sink_size if causal else 0, st.window_size if causal else 0))
        with gm.graph.inserting_before(hit.out):
            repl = gm.graph.call_module(name, args=(hit.q, hit.k, hit.v))
        hit.out.replace_all_uses_with(repl)
        for dead in (hit.out, hit.softmax, hit.scaled, hit.scores, hit.kt):
            if dead is not None:
                _erase_if_dead(gm.graph, dead)


def pretty_print_graph(gm: fx.GraphModule, header: str = "") -> str:
    """Generated code of ``gm`` plus a tally of node kinds."""
    lines = [f"=== {header} ==="] if header else []
    lines.append(gm.graph.python_code(root_module="self").src.strip())
    tally: dict = {}
    for n in gm.graph.nodes:
        tally[n.op] = tally.get(n.op, 0) + 1
    lines.append("# node tally: " + ", ".join(f"{k}={v}" for k, v in sorted(tally.items())))
    return "\n".join(lines)


__all__ = [
    "BlockSparseAttentionInjector",
    "InjectionConfig",
    "SingleLayerTransformer",
    "StandardAttention",
    "pretty_print_graph",
]
