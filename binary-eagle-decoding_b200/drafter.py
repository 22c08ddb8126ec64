"""Block-drafter forward engine for the B200: HE4.forward of the reference as a
device-resident, CUDA-graph-capturable draft step.

Follows ``w1a1_eagle/model.py``: ``HE4.forward`` (369-396), ``Layer.context``
(195-200) and ``Layer.forward`` (202-223).  The reference recomputes the fused
context and every layer's context K/V on each call; the engine keeps them in an
fp16 K/V cache (exactly the values ``cache_storage`` would produce) filled by
``prefill`` and extended by ``ingest``, so a draft round reads each weight once.

Device data (all on one GPU):
  * dense matrices (fc, per-layer q|k|v and o, the tied vocabulary) as bf16
    W16 tiles for ``bd_gemv_bf16``; the vocabulary also as a plain bf16 table
    for the embedding gather;
  * the one-bit feed-forward blocks as T16 sign tiles with fp32 scales,
    midpoints and exponentiated gains/clip bounds (``ops.PackedFFN``);
  * K/V caches fp16 ``[layers][positions][kv_heads][head_dim]``.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

from . import _lib, ops
from .ops import Flags, PackedFFN, _p, _stream


def _w16(weight: Tensor) -> Tensor:
    """W16 tiles (uint8 storage) of a row-major fp32/bf16 matrix."""
    weight = weight.contiguous()
    rows, cols = weight.shape
    out = torch.empty(int(_lib.load().bd_w16_bytes(rows, cols)), dtype=torch.uint8, device=weight.device)
    bits = 32 if weight.dtype == torch.float32 else 16
    if weight.dtype not in (torch.float32, torch.bfloat16):
        weight = weight.float()
        bits = 32
    _lib.call("bd_tile_w16", _p(weight), bits, rows, cols, _p(out), _stream(weight.device))
    return out


@dataclass
class LayerDevice:
    qkv: Tensor            # W16 of cat(attn_q, attn_k, attn_v)
    o: Tensor              # W16 of attn_output
    attn_norm: Tensor
    q_norm: Tensor
    k_norm: Tensor
    ffn_norm: Tensor
    ffn: PackedFFN


class DraftEngine:
    """One drafter on one device.  ``tokens`` per call (block slots) <= 32."""

    def __init__(self, tensors: dict[str, Tensor], vocabulary: Tensor, mask: int, geometry, quantizers: dict | None = None,
                 device: torch.device | str = "cuda", max_positions: int | None = None):
        cfg = self.cfg = geometry
        self.device = torch.device(device)
        self.mask = int(mask)
        self.vocab_size, hidden = vocabulary.shape
        if hidden != cfg.hidden:
            raise ValueError("invalid frozen vocabulary geometry or mask")
        self.max_positions = int(max_positions or (cfg.window + cfg.slots))
        dev = self.device

        def t(name):
            return tensors[name].to(dev)

        vocab = vocabulary.to(dev)
        self.vocab16 = vocab.to(torch.bfloat16).contiguous()
        self.head = _w16(self.vocab16)
        self.fc = _w16(t("fc.weight").to(torch.bfloat16))
        self.fc_bf16 = t("fc.weight").to(torch.bfloat16).contiguous()
        self.enc_norm = t("enc.output_norm.weight").float().contiguous()
        self.out_norm = t("output_norm.weight").float().contiguous()
        quantizers = quantizers or {}
        self.layers: list[LayerDevice] = []
        self.kv_bf16: list[Tensor] = []
        self.kv_bf16x2: list[Tensor] = []  # [K | K] for the hi + lo product of a prefill
        for i in range(cfg.layers):
            p = f"blk.{i}."
            q, k, v = t(p + "attn_q.weight"), t(p + "attn_k.weight"), t(p + "attn_v.weight")
            qkv = torch.cat((q, k, v), 0).to(torch.bfloat16)
            self.kv_bf16.append(torch.cat((k, v), 0).to(torch.bfloat16).contiguous())
            self.kv_bf16x2.append(torch.cat((self.kv_bf16[-1], self.kv_bf16[-1]), 1).contiguous())
            gate, up, down = t(p + "ffn_gate.weight").float(), t(p + "ffn_up.weight").float(), t(p + "ffn_down.weight").float()

            def qv(name, default):
                value = quantizers.get(p + name)
                return (default if value is None else value.to(dev).float()).contiguous().reshape(-1)

            ffn = ops.pack_ffn(gate, up, down, qv("ffn_gate.scale", gate.abs().mean(-1)),
                               qv("ffn_up.scale", up.abs().mean(-1)), qv("ffn_down.scale", down.abs().mean(-1)))
            ffn.midpoint_gate = qv("ffn_gate.midpoint", torch.zeros(cfg.intermediate, device=dev))
            ffn.midpoint_up = qv("ffn_up.midpoint", torch.zeros(cfg.intermediate, device=dev))
            ffn.midpoint_down = qv("ffn_down.midpoint", torch.zeros(cfg.hidden, device=dev))
            ffn.gain_gate_up = qv("ffn_gate_up.gain", torch.ones(cfg.hidden, device=dev))
            ffn.bound_gate_up = qv("ffn_gate_up.bound", torch.ones(1, device=dev))
            ffn.gain_down = qv("ffn_down.gain", torch.ones(cfg.intermediate, device=dev))
            ffn.bound_down = qv("ffn_down.bound", torch.ones(1, device=dev))
            self.layers.append(LayerDevice(
                qkv=_w16(qkv), o=_w16(t(p + "attn_output.weight").to(torch.bfloat16)),
                attn_norm=t(p + "attn_norm.weight").float().contiguous(), q_norm=t(p + "attn_q_norm.weight").float().contiguous(),
                k_norm=t(p + "attn_k_norm.weight").float().contiguous(), ffn_norm=t(p + "ffn_norm.weight").float().contiguous(),
                ffn=ffn))
        kvd = cfg.kv_heads * cfg.head_dim
        # every layer's k|v rows stacked: the context rows of an ingest step are one
        # GEMV over all layers (they share the encoded input)
        self.kv_all = _w16(torch.cat(self.kv_bf16, 0))
        self.k_norms = torch.stack([layer.k_norm for layer in self.layers]).contiguous()
        self.k_cache = torch.zeros((cfg.layers, self.max_positions, kvd), dtype=torch.float16, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.qkv_width = (cfg.heads + 2 * cfg.kv_heads) * cfg.head_dim
        # per-call buffers (fixed addresses, so a draft step can be captured in a graph)
        T = 32
        self.ids = torch.zeros(T, dtype=torch.int32, device=dev)
        self.state = torch.zeros((T, cfg.hidden), dtype=torch.float32, device=dev)
        self.resid = torch.zeros_like(self.state)
        self.normed = torch.zeros_like(self.state)
        self.qkv_out = torch.zeros((T, self.qkv_width), dtype=torch.float32, device=dev)
        self.q_rows = torch.zeros((T, cfg.heads * cfg.head_dim), dtype=torch.float32, device=dev)
        widest = max(cfg.hidden, cfg.heads * cfg.head_dim, cfg.taps * cfg.hidden)
        self.x16 = torch.zeros(int(_lib.load().bd_x16_bytes(T, widest)), dtype=torch.uint8, device=dev)
        # the ingest step packs into its own buffer, so a round can run it beside the
        # draft's first kernels (only the context fusion splits K over the shared GEMV
        # workspace; no draft GEMV does)
        self.x16_ctx = torch.zeros_like(self.x16)
        self.keys = torch.zeros(T, dtype=torch.int64, device=dev)
        self.drafted = torch.zeros(T, dtype=torch.int32, device=dev)
        self.encoded = torch.zeros((T, cfg.hidden), dtype=torch.float32, device=dev)
        self.fused = torch.zeros((T, cfg.hidden), dtype=torch.float32, device=dev)
        self.kv_out = torch.zeros((T, cfg.layers * 2 * kvd), dtype=torch.float32, device=dev)
        if cfg.head_dim not in (64, 128) or cfg.heads // cfg.kv_heads > 4 or cfg.slots > 16:
            raise ValueError("attention kernel geometry: head_dim 64/128, at most 4 q heads per kv head, <= 16 slots")
        self.attn_ws = torch.zeros(int(_lib.load().bd_attention_workspace_bytes(cfg.heads, cfg.head_dim,
                                                                                 self.max_positions)),
                                   dtype=torch.uint8, device=dev)
        lib = _lib.load()
        shapes = [(cfg.hidden, cfg.taps * cfg.hidden), (cfg.layers * 2 * kvd, cfg.hidden), (self.qkv_width, cfg.hidden),
                  (cfg.hidden, cfg.heads * cfg.head_dim), (self.vocab_size, cfg.hidden)]
        self.gemv_ws = torch.zeros(max(256, max(int(lib.bd_gemv_workspace_bytes(T, r, c)) for r, c in shapes)),
                                   dtype=torch.uint8, device=dev)
        self.flags = Flags(dev)
        self.positions = 0

    # ------------------------------------------------------------------ helpers
    def _stream(self) -> int:
        return _stream(self.device)

    def _pack(self, x: Tensor, n: int, cols: int, ld: int, weight: Tensor | None = None, normed: Tensor | None = None,
              x16: Tensor | None = None):
        _lib.call("bd_pack_x16", _p(x), n, cols, ld, _p(weight), float(self.cfg.epsilon),
                  _p(self.x16 if x16 is None else x16), _p(normed), normed.shape[1] if normed is not None else 0,
                  self.flags.ptr, self._stream())

    def _gemv(self, w16_ptr: int, rows: int, cols: int, n: int, out: Tensor | None, ld_out: int,
              residual: Tensor | None = None, keys: Tensor | None = None, x16: Tensor | None = None):
        _lib.call("bd_gemv_bf16", w16_ptr, rows, cols, _p(self.x16 if x16 is None else x16), n, _p(out), ld_out,
                  _p(residual), _p(keys), self.flags.ptr, _p(self.gemv_ws), self.gemv_ws.numel(), self._stream())

    def _heads(self, src: Tensor, n: int, col0: int, heads: int, norm: Tensor | None, rope: bool, pos0: int,
               dst_ptr: int, dst_ld: int):
        cfg = self.cfg
        _lib.call("bd_heads_post", _p(src), n, src.shape[1], col0, heads, cfg.head_dim, _p(norm), float(cfg.epsilon),
                  int(rope), float(cfg.theta), pos0, dst_ptr, dst_ld, self.flags.ptr, self._stream())

    def _cache_ptr(self, cache: Tensor, layer: int, pos: int) -> int:
        return cache[layer, pos].data_ptr()

    def check(self) -> None:
        """Raise the reference's ValueError for any device-reported condition."""
        self.flags.check()

    # ------------------------------------------------------------------ context
    def prefill(self, features: Tensor, anchor: int) -> None:
        """Context K/V of positions [0, anchor) from target features (model.py:382-386, 195-200).

        The fusion and context K/V products run on the tensor cores
        (``bd_gemm_bf16``: tcgen05 bf16 MMAs, fp32 accumulators in TMEM); the
        K/V product takes the encoded rows as bf16 hi + lo halves along K, the
        same ~16-bit split the GEMV path uses.  Normalisation, rotary embedding
        and fp16 storage are this library's kernels.
        """
        cfg = self.cfg
        if anchor > self.max_positions - cfg.slots:
            raise ValueError("context longer than the engine's cache")
        self.positions = anchor
        if anchor == 0:
            return
        feats = features[:anchor].to(self.device, torch.bfloat16).contiguous()
        fused = ops.gemm_bf16(feats, self.fc_bf16)
        encoded = torch.empty_like(fused)
        _lib.call("bd_rms_rows", _p(fused), anchor, cfg.hidden, cfg.hidden, _p(self.enc_norm), float(cfg.epsilon),
                  _p(encoded), cfg.hidden, self._stream())
        # encoded rows as bf16 hi + lo (the same ~16-bit split the GEMV path uses), side by side along K
        enc_hi = encoded.to(torch.bfloat16)
        enc = torch.cat((enc_hi, (encoded - enc_hi.float()).to(torch.bfloat16)), 1).contiguous()
        kvd = cfg.kv_heads * cfg.head_dim
        for i, layer in enumerate(self.layers):
            kv = ops.gemm_bf16(enc, self.kv_bf16x2[i])
            self._heads(kv, anchor, 0, cfg.kv_heads, layer.k_norm, True, 0, self._cache_ptr(self.k_cache, i, 0), kvd)
            self._heads(kv, anchor, kvd, cfg.kv_heads, None, False, 0, self._cache_ptr(self.v_cache, i, 0), kvd)

    def ingest(self, features: Tensor, pos0: int, after_fusion=None) -> None:
        """Append up to 32 context rows at positions pos0.. through the GEMV path (one draft
        round).  ``after_fusion`` (optional) is called once the fusion GEMV is issued."""
        cfg = self.cfg
        n = features.shape[0]
        if not 1 <= n <= 32 or pos0 + n > self.max_positions - cfg.slots:
            raise ValueError("invalid context rows")
        width = cfg.taps * cfg.hidden
        x16 = self.x16_ctx
        if features.dtype == torch.bfloat16 and features.is_cuda and features.is_contiguous():
            # bf16 rows pack straight into X16 (the same bits as their fp32 values)
            _lib.call("bd_pack_x16_bf16", _p(features), n, width, width, None, float(cfg.epsilon), _p(x16), None, 0,
                      self.flags.ptr, self._stream())
        else:
            feats = features if features.dtype == torch.float32 else features.float()
            self._pack(feats.to(self.device).contiguous(), n, width, width, x16=x16)
        self._gemv(self.fc.data_ptr(), cfg.hidden, width, n, self.fused, cfg.hidden, x16=x16)
        if after_fusion is not None:
            after_fusion()
        self._pack(self.fused, n, cfg.hidden, cfg.hidden, self.enc_norm, x16=x16)
        kvd = cfg.kv_heads * cfg.head_dim
        width_kv = cfg.layers * 2 * kvd
        self._gemv(self.kv_all.data_ptr(), width_kv, cfg.hidden, n, self.kv_out, width_kv, x16=x16)
        _lib.call("bd_context_kv_post", _p(self.kv_out), n, width_kv, cfg.layers, 2 * kvd, cfg.kv_heads, cfg.head_dim,
                  _p(self.k_norms), float(cfg.epsilon), float(cfg.theta), pos0, self._cache_ptr(self.k_cache, 0, pos0),
                  self._cache_ptr(self.v_cache, 0, pos0), kvd, self.max_positions * kvd, self.flags.ptr,
                  self._stream())
        self.positions = max(self.positions, pos0 + n)

    # ------------------------------------------------------------------ draft
    def set_tokens(self, first: int, size: int) -> None:
        ids = torch.full((size,), self.mask, dtype=torch.int32)
        ids[0] = first
        self.ids[:size].copy_(ids, non_blocking=True)

    def embed(self, k: int) -> None:
        """``state[:k]`` = embedding rows of ``ids[:k]`` (model.py:380-381)."""
        _lib.call("bd_embed_rows", _p(self.vocab16), self.vocab_size, self.cfg.hidden, _p(self.ids), k,
                  _p(self.state), self.flags.ptr, self._stream())

    def attention_half(self, i: int, anchor: int, k: int) -> None:
        """``resid[:k] = state + o(attention)`` of layer i (model.py:202-219); the block's
        K/V rows go to cache positions anchor.."""
        self.qkv_rows(i, anchor, k)
        self.attend(i, anchor, k)

    def qkv_rows(self, i: int, anchor: int, k: int) -> None:
        """q rows of layer i and the block's K/V cache rows at anchor.. (model.py:202-213)."""
        cfg = self.cfg
        layer = self.layers[i]
        H, qd, kvd = cfg.hidden, cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
        self._pack(self.state, k, H, H, layer.attn_norm)
        self._gemv(layer.qkv.data_ptr(), self.qkv_width, H, k, self.qkv_out, self.qkv_width)
        _lib.call("bd_qkv_post", _p(self.qkv_out), k, self.qkv_width, cfg.heads, cfg.kv_heads, cfg.head_dim,
                  _p(layer.q_norm), _p(layer.k_norm), float(cfg.epsilon), float(cfg.theta), anchor,
                  _p(self.q_rows), qd, self._cache_ptr(self.k_cache, i, anchor),
                  self._cache_ptr(self.v_cache, i, anchor), kvd, self.flags.ptr, self._stream())

    def attend(self, i: int, anchor: int, k: int) -> None:
        """``resid[:k] = state + o(attention)`` from the q rows and the cache (model.py:212-219)."""
        cfg = self.cfg
        H, qd = cfg.hidden, cfg.heads * cfg.head_dim
        layer = self.layers[i]
        st = self._stream()
        windowed = int(i < cfg.layers - 1)
        # rows below the anchor were written by the ingest step, several kernels earlier;
        # the attention writes its rows as the output projection's X16 activations
        _lib.call("bd_attention_decode_x16", _p(self.q_rows), self._cache_ptr(self.k_cache, i, 0),
                  self._cache_ptr(self.v_cache, i, 0), k, cfg.heads, cfg.kv_heads, cfg.head_dim, anchor + k,
                  windowed, anchor, cfg.window, anchor, _p(self.x16), self.flags.ptr, _p(self.attn_ws),
                  self.attn_ws.numel(), st)
        self._gemv(layer.o.data_ptr(), H, qd, k, self.resid, H, residual=self.state)

    def ffn_half(self, i: int, k: int) -> None:
        """``state[:k] = resid + ffn(rms(resid))`` of layer i (model.py:220-223)."""
        layer = self.layers[i]
        ops.ffn_he4(self.resid[:k], layer.ffn, self.resid[:k], flags=self.flags, out=self.state[:k],
                    norm=layer.ffn_norm, epsilon=self.cfg.epsilon)

    def draft_start(self, anchor: int, size: int | None = None) -> None:
        """The part of a block that reads no context row: the slot embeddings and layer
        0's q|k|v rows (the block's own K/V cache rows)."""
        k = self.cfg.slots if size is None else size
        self.embed(k)
        self.qkv_rows(0, anchor, k)

    def draft(self, anchor: int, size: int | None = None, logits: Tensor | None = None, join=None,
              started: bool = False) -> Tensor:
        """One block of the drafter over the cached context (model.py:369-396).

        Slot tokens come from ``self.ids`` (``set_tokens``); returns the argmax
        token of every slot (int32 [size], device) and fills ``logits`` [size, V]
        when given.  Graph-capturable for fixed (anchor, size).  ``join(i)`` (optional) is
        called after layer i's q|k|v rows and before its attention, the first kernel
        that reads layer i's cache rows below the anchor: a round that ingests context
        rows on other streams waits for them there.  ``started``: ``draft_start``
        already ran (on another stream, joined before this call).
        """
        cfg = self.cfg
        k = cfg.slots if size is None else size
        H = cfg.hidden
        st = self._stream()
        if not started:
            self.draft_start(anchor, k)
        for i in range(len(self.layers)):
            if i > 0:
                self.qkv_rows(i, anchor, k)
            if join is not None:
                join(i)  # the context rows the attention reads are complete from here on
            self.attend(i, anchor, k)
            self.ffn_half(i, k)
        self._pack(self.state, k, H, H, self.out_norm)
        self._gemv(self.head.data_ptr(), self.vocab_size, H, k, logits, self.vocab_size, keys=self.keys)
        _lib.call("bd_argmax_finish", _p(self.keys), k, _p(self.drafted), st)
        return self.drafted[:k]


class DraftRound:
    """A captured draft round: ingest ``rows`` new context rows ending at ``anchor``,
    then draft a block of ``size`` slots.  ``__call__`` is the serving entry point:
    host (pinned) rows and the anchor token in, drafted tokens (slots 1..size-1) out.
    """

    def __init__(self, engine: DraftEngine, anchor: int, size: int, rows: int):
        cfg = engine.cfg
        self.engine, self.anchor, self.size, self.rows = engine, anchor, size, rows
        dev = engine.device
        width = cfg.taps * cfg.hidden
        self.dev_rows = torch.zeros((rows, width), dtype=torch.bfloat16, device=dev)
        self.host_rows = torch.zeros((rows, width), dtype=torch.bfloat16).pin_memory()
        self.host_first = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.host_out = torch.zeros(size, dtype=torch.int32).pin_memory()
        engine.set_tokens(engine.mask, size)
        # the ingest (on the capture stream) gates layer 0's attention: the higher priority
        self.stream = torch.cuda.Stream(dev, priority=-1)
        self.side = torch.cuda.Stream(dev)
        self.stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(self.stream):
            for _ in range(2):
                self._body()
        self.stream.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self._body()
        # the served round: the same work with its host copies inside the graph, the
        # rows' host-to-device copy on the ingest's stream beside the draft's first kernels
        self.served = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.served, stream=self.stream):
            self._body(host=True)
        self.stream.synchronize()
        engine.check()

    def _body(self, host: bool = False) -> None:
        # the ingest step (fusion + context k|v of the new rows) runs beside the draft's
        # embedding and layer-0 q|k|v rows, which do not read the context; the ingest,
        # the longer of the two, is on the capture stream, whose kernels the graph
        # launches first
        e = self.engine
        main = torch.cuda.current_stream(e.device)
        if host:
            e.ids[:1].copy_(self.host_first, non_blocking=True)
            self.dev_rows.copy_(self.host_rows, non_blocking=True)

        def fork() -> None:
            # the draft's first kernels start once the fusion GEMV (the widest read) is issued
            self.side.wait_stream(main)
            with torch.cuda.stream(self.side):
                e.draft_start(self.anchor, self.size)

        e.ingest(self.dev_rows, self.anchor - self.rows, after_fusion=fork)
        main.wait_stream(self.side)
        e.draft(self.anchor, self.size, started=True)
        if host:
            self.host_out.copy_(e.drafted[: self.size], non_blocking=True)

    def replay(self) -> None:
        self.graph.replay()

    @property
    def h2d_bytes(self) -> int:
        return self.host_rows.numel() * self.host_rows.element_size() + 4

    @property
    def d2h_bytes(self) -> int:
        return self.size * 4

    def __call__(self, first_token: int | None = None) -> Tensor:
        """H2D of ``host_rows`` (+ the anchor token), one round, D2H of the drafted tokens
        (``bd_round_submit``: one launch of the served graph, which holds the copies,
        and the wait, in one C call)."""
        if first_token is not None:
            self.host_first[0] = first_token
        _lib.call("bd_round_submit", self.served.raw_cuda_graph_exec(), None, None, 0, None, None, None, None, 0,
                  self.stream.cuda_stream, kernels=0)
        return self.host_out[1:]
