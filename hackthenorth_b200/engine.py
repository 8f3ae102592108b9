"""Drop-in ``Engine`` for the dryft Qwen3 decode path on sm_100a kernels: batch
one (speculative with prompt lookup by default, as the reference), and batched
decode of any number of equal-length prompts (8 per context per step).

Public API (``dryft/QWEN_ENGINE_CONTRACT.md:25-36``, ``dryft/engine/engine.py:175-249``):

    engine = Engine(model_path)                       # HF checkpoint directory
    for step in engine.generate(input_ids, max_new_tokens):
        ...                                           # step == [token_id]

``generate`` yields one token id per sequence exactly ``max_new_tokens``
times and never stops at an end-of-sequence token. The internal entry points the north
star names map as follows: load = ``Engine.__init__``; prefill =
``DecodeState.prefill``; decode_step = ``DecodeState.step`` (a replay of the
captured graph); generate = ``Engine.generate``.

PyTorch owns device memory and streams; every kernel is in ``libqb.so``.
"""
from __future__ import annotations

from typing import Dict, Iterator, List, Optional

import torch

from . import _lib
from .config import ModelConfig
from .weights import PackedWeights, load_checkpoint, random_state_dict, rotary_table

BF16 = torch.bfloat16


class _TokenHandle:
    """A decode step's tokens on their way to the host: a pinned ring slot
    filled by an asynchronous device-to-host copy, and the event after it."""

    __slots__ = ("host", "event")

    def __init__(self, host, event):
        self.host, self.event = host, event

    def result(self) -> List[int]:
        self.event.synchronize()
        return self.host.tolist()


def stream_decode(state, first_tokens: List[int], output_length: int, depth: int = 1) -> Iterator[List[int]]:
    """Overlap graph replays with the delivery of tokens already read
    (``dryft/engine/decode.py:8-22``): the final yield has no outstanding replay
    and ``output_length == 1`` launches none.

    ``depth`` 1 is the reference's order (the next replay is launched, the
    current token yielded, then the new token read synchronously). With
    ``depth`` d > 1 and a state offering ``read_token_async`` (a device-to-host
    token ring), up to d replays run ahead of the consumer: each replay's
    tokens are copied asynchronously into a pinned slot, and a yield waits
    only for its own step, so the GPU never idles between steps while the
    host converts and yields."""
    if depth <= 1 or not hasattr(state, "read_token_async"):
        tokens = first_tokens
        for step in range(output_length):
            has_next = step + 1 < output_length
            if has_next:
                state.step()
            yield tokens
            if has_next:
                tokens = state.read_token()
        return
    from collections import deque

    pending = deque()
    issued = 0
    total = output_length - 1  # replays needed

    def launch():
        nonlocal issued
        state.step()
        pending.append(state.read_token_async(depth + 1))
        issued += 1

    while issued < min(depth, total):
        launch()
    if output_length >= 1:
        yield first_tokens
    for _ in range(total):
        handle = pending.popleft()
        if issued < total:
            launch()
        yield handle.result()


class DecodeState:
    """Fixed-capacity KV cache, RoPE table, device token/position and the
    captured decode graph (``dryft/engine/decode.py:102-206``).

    Capacity = prompt_length + output_length - 1 + draft slots. The caches are
    zero-filled (finite), laid out ``[L, Hkv, capacity, D]``; with ``batch`` B > 1
    sequences (one GPU, B <= 8) ``[L, B, Hkv, capacity, D]``, and ``token`` /
    ``position`` hold one entry per sequence.
    """

    MAX_BATCH = 8

    def __init__(self, engine: "Engine", prompt_length: int, output_length: int,
                 draft_tokens: int = 0, keep_logits: bool = False, capacity: Optional[int] = None,
                 batch: int = 1):
        cfg = engine.cfg
        dev = engine.device
        if not 1 <= batch <= self.MAX_BATCH:
            raise ValueError(f"batch must lie in 1..{self.MAX_BATCH}")
        if batch > 1 and engine.tp_size > 1:
            raise ValueError("batched decode runs on one GPU")
        self.engine = engine
        self.batch = batch
        self.draft_tokens = draft_tokens
        self.shape = (batch, prompt_length, output_length)
        self.capacity = capacity or (prompt_length + max(output_length, 1) - 1 + draft_tokens)
        hkv = cfg.n_kv_heads // engine.tp_size
        shape = ((cfg.n_layers, hkv, self.capacity, cfg.head_dim) if batch == 1
                 else (cfg.n_layers, batch, hkv, self.capacity, cfg.head_dim))
        self.keys = torch.zeros(shape, dtype=BF16, device=dev)
        self.values = torch.zeros(shape, dtype=BF16, device=dev)
        cos, sin = rotary_table(cfg, self.capacity)
        self.cos, self.sin = cos.to(dev), sin.to(dev)
        L = _lib.load()
        nbytes = _lib.c_size_t()
        _lib.check(L.qb_workspace_bytes(engine.ctx, _lib.ctypes.byref(nbytes)), engine.ctx)
        self.workspace = torch.empty(nbytes.value, dtype=torch.uint8, device=dev)
        self.token = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.position = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.prompt = torch.zeros(batch * max(prompt_length, 1), dtype=torch.int64, device=dev)
        # this rank's vocabulary shard under tensor parallelism; [B, V] batched
        vshape = (cfg.vocab // engine.tp_size,) if batch == 1 else (batch, cfg.vocab)
        self.logits = torch.zeros(vshape, dtype=BF16, device=dev) if keep_logits else None
        _lib.check(L.qb_set_batch(engine.ctx, batch), engine.ctx)
        _lib.check(L.qb_bind_state(engine.ctx, self.keys.data_ptr(), self.values.data_ptr(), self.capacity,
                                   self.cos.data_ptr(), self.sin.data_ptr(), self.workspace.data_ptr(),
                                   self.workspace.numel()), engine.ctx)
        engine._bound_state = self
        self.captured = False

    # -- the four entry points --------------------------------------------------
    # Prompts of at least this many rows run as dense blocks (tensor-core
    # GEMMs and flash attention); shorter ones through the decode kernels.
    BATCHED_PREFILL_MIN = 8

    def prefill(self, ids: torch.Tensor, batched: Optional[bool] = None) -> torch.Tensor:
        """Write K/V for the prompt, emit the first token into ``self.token``
        and set ``position = len(prompt)``. ``batched`` forces (True) or
        forbids (False) the dense-block path; by default it is used for
        prompts of ``BATCHED_PREFILL_MIN`` rows or more (under tensor
        parallelism too: every rank calls it with the same prompt). With
        ``batch`` B > 1, ``ids`` is ``[B, P]`` (equal prompt lengths) and the
        prompts run as P teacher-forced batched passes."""
        if self.batch > 1:
            if ids.dim() != 2 or ids.shape[0] != self.batch:
                raise ValueError(f"batched prefill takes ids of shape [{self.batch}, P]")
            if batched:
                raise ValueError("the dense-block prefill takes one sequence")
            batched = False
        n = ids.shape[-1] if self.batch > 1 else ids.numel()
        if n > self.capacity:
            raise ValueError("prompt longer than the KV capacity")
        if self.batch * n > self.prompt.numel():
            self.prompt = torch.zeros(self.batch * n, dtype=torch.int64, device=self.token.device)
        self.prompt[:self.batch * n].copy_(ids.reshape(-1), non_blocking=True)
        self._ensure_bound()
        L = _lib.load()
        if batched is None:
            batched = n >= self.BATCHED_PREFILL_MIN
        if batched:
            need = _lib.c_size_t()
            _lib.check(L.qb_prefill_scratch_bytes(self.engine.ctx, n, _lib.ctypes.byref(need)), self.engine.ctx)
            scratch = getattr(self, "_prefill_scratch", None)
            if scratch is None or scratch.numel() < need.value:
                self._prefill_scratch = scratch = torch.empty(need.value, dtype=torch.uint8,
                                                              device=self.token.device)
            _lib.check(L.qb_prefill_batched(self.engine.ctx, self.prompt.data_ptr(), n, scratch.data_ptr(),
                                            scratch.numel(), self.token.data_ptr(), self.position.data_ptr(),
                                            _lib.ptr(self.logits), _lib.stream_handle()), self.engine.ctx)
        else:
            _lib.check(L.qb_prefill(self.engine.ctx, self.prompt.data_ptr(), n, self.token.data_ptr(),
                                    self.position.data_ptr(), _lib.ptr(self.logits), _lib.stream_handle()),
                       self.engine.ctx)
        return self.token

    def capture(self) -> None:
        """Capture one decode step as a CUDA graph on a side stream."""
        self._ensure_bound()
        side = torch.cuda.Stream(device=self.token.device)
        side.wait_stream(torch.cuda.current_stream())
        _lib.check(_lib.load().qb_capture_decode(self.engine.ctx, self.token.data_ptr(), self.position.data_ptr(),
                                                 _lib.ptr(self.logits), side.cuda_stream), self.engine.ctx)
        torch.cuda.current_stream().wait_stream(side)
        self.captured = True

    def step(self) -> None:
        """One decode step: token <- greedy(next), position += 1."""
        self._ensure_bound()
        if not self.captured:
            self.capture()
        _lib.check(_lib.load().qb_replay_decode(self.engine.ctx, _lib.stream_handle()), self.engine.ctx)

    def step_eager(self) -> None:
        self._ensure_bound()
        _lib.check(_lib.load().qb_decode_step(self.engine.ctx, self.token.data_ptr(), self.position.data_ptr(),
                                              _lib.ptr(self.logits), _lib.stream_handle()), self.engine.ctx)

    def read_token(self) -> List[int]:
        return self.token.tolist()

    def read_token_async(self, slots: int = 3) -> _TokenHandle:
        """Queue a device-to-host copy of ``token`` (after the work queued so
        far on the current stream) into the next of ``slots`` pinned host
        slots; ``.result()`` waits for that copy only."""
        ring = getattr(self, "_token_ring", None)
        if ring is None or len(ring) != slots:
            ring = [(torch.empty(self.batch, dtype=torch.int64).pin_memory(), torch.cuda.Event())
                    for _ in range(slots)]
            self._token_ring, self._ring_next = ring, 0
        host, event = ring[self._ring_next % slots]
        self._ring_next += 1
        host.copy_(self.token, non_blocking=True)
        event.record()
        return _TokenHandle(host, event)

    def check(self) -> None:
        """Synchronise and raise on a device-side error (bounded wait gave up,
        token or position out of range)."""
        _lib.check(_lib.load().qb_check(self.engine.ctx, _lib.stream_handle()), self.engine.ctx)

    # -- speculative verification ------------------------------------------------
    def verify(self, current_token: int, proposal: List[int]) -> List[int]:
        """Verify ``proposal`` after ``current_token`` (``DecodeState.verify``,
        ``dryft/engine/decode.py:194-206``): the ``len(proposal) + 1`` rows run
        at positions ``position ..`` in one pass (a captured graph per row
        count), the accepted prefix plus one target token is returned, and
        ``token`` / ``position`` advance by that many; the K/V of rejected
        rows stay in the cache as dead slots that later steps overwrite."""
        from .speculate import verified_tokens

        self._ensure_bound()
        if self.batch > 1:
            raise ValueError("verify takes one sequence")
        n = len(proposal) + 1
        if n > 8:
            raise ValueError("verify takes at most 7 draft tokens")
        dev = self.token.device
        if getattr(self, "_verify_n", None) != n:
            if not hasattr(self, "verify_ids"):
                self.verify_ids = torch.zeros(8, dtype=torch.int64, device=dev)
                self.verify_out = torch.zeros(8, dtype=torch.int64, device=dev)
                self._verify_host = torch.zeros(8, dtype=torch.int64).pin_memory()
            self.verify_logits = (torch.zeros(n, self.engine.cfg.vocab // self.engine.tp_size, dtype=BF16, device=dev)
                                  if self.logits is not None else None)
            side = torch.cuda.Stream(device=dev)
            side.wait_stream(torch.cuda.current_stream())
            _lib.check(_lib.load().qb_capture_verify(self.engine.ctx, self.verify_ids.data_ptr(), n,
                                                     self.position.data_ptr(), self.verify_out.data_ptr(),
                                                     _lib.ptr(self.verify_logits), side.cuda_stream),
                       self.engine.ctx)
            torch.cuda.current_stream().wait_stream(side)
            self._verify_n = n
        self._verify_host[:n] = torch.tensor([current_token, *proposal], dtype=torch.int64)
        self.verify_ids[:n].copy_(self._verify_host[:n], non_blocking=True)
        _lib.check(_lib.load().qb_replay_verify(self.engine.ctx, _lib.stream_handle()), self.engine.ctx)
        predictions = self.verify_out[:n].tolist()
        emitted = verified_tokens(proposal, predictions)
        self.token.fill_(emitted[-1])
        self.position.add_(len(emitted))
        return emitted

    def _ensure_bound(self):
        if self.engine._bound_state is not self:
            raise RuntimeError("this DecodeState is no longer bound to its engine")


class Engine:
    """``Engine(model_path)``: load an HF Qwen3 checkpoint to ``cuda:0`` in the
    engine layout; ``generate`` streams greedy tokens."""

    # decode replays in flight ahead of the consumer in ``generate``
    STREAM_DEPTH = 2

    def __init__(self, model_path: Optional[str] = None, device: str = "cuda:0", *,
                 cfg: Optional[ModelConfig] = None, state: Optional[Dict[str, torch.Tensor]] = None,
                 tp_rank: int = 0, tp_size: int = 1, unique_id: Optional[bytes] = None):
        """``tp_rank``/``tp_size``: tensor-parallel slot (one process per GPU);
        every rank of the group passes the same ``unique_id`` (from
        ``hackthenorth_b200.tp.unique_id`` on rank 0, shared by the caller)."""
        if not torch.cuda.is_available():
            raise RuntimeError("Engine needs a CUDA device; there is no CPU fallback")
        self.device = torch.device(device)
        torch.cuda.set_device(self.device)
        if model_path is not None:
            cfg, state = load_checkpoint(model_path, device="cpu")
        if cfg is None or state is None:
            raise ValueError("Engine needs a model_path or (cfg, state)")
        self.cfg = cfg
        self.tp_rank, self.tp_size = tp_rank, tp_size
        self.weights = PackedWeights(cfg, state, self.device, tp_rank, tp_size)
        L = _lib.load()
        qc = _lib.QbConfig(cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn, cfg.n_layers,
                           cfg.vocab, cfg.rms_eps)
        ctx = _lib.c_void_p()
        _lib.check(L.qb_create(_lib.ctypes.byref(qc), self.device.index or 0, tp_rank, tp_size,
                               _lib.ctypes.byref(ctx)))
        self.ctx = ctx
        if tp_size > 1:
            if unique_id is None:
                raise ValueError("tensor parallelism needs the group's NCCL unique id")
            buf = _lib.ctypes.create_string_buffer(bytes(unique_id), len(unique_id))
            _lib.check(L.qb_tp_init(ctx, buf), ctx)
        table = (_lib.QbLayerWeights * cfg.n_layers)()
        for i, lw in enumerate(self.weights.layers):
            table[i] = _lib.QbLayerWeights(lw["input_norm"].data_ptr(), lw["qkv"].data_ptr(),
                                           lw["q_norm"].data_ptr(), lw["k_norm"].data_ptr(), lw["o"].data_ptr(),
                                           lw["post_norm"].data_ptr(), lw["gu"].data_ptr(), lw["down"].data_ptr())
        w = self.weights
        _lib.check(L.qb_bind_weights(ctx, table, cfg.n_layers, w.embed.data_ptr(), w.final_norm.data_ptr(),
                                     w.lm_head.data_ptr()), ctx)
        if tp_size > 1:
            # the block prefill's column-parallel o-proj and down (row shards)
            o_rows = (_lib.c_void_p * cfg.n_layers)(*[lw["o_rows"].data_ptr() for lw in w.layers])
            down_rows = (_lib.c_void_p * cfg.n_layers)(*[lw["down_rows"].data_ptr() for lw in w.layers])
            _lib.check(L.qb_bind_prefill_weights(ctx, o_rows, down_rows, cfg.n_layers), ctx)
        self._weight_table = table
        self.state: Optional[DecodeState] = None
        self._bound_state = None
        self._lanes: List["_Lane"] = []

    @classmethod
    def from_random(cls, cfg: ModelConfig, seed: int = 0, device: str = "cuda:0", init_device: str = "cpu",
                    tp_rank: int = 0, tp_size: int = 1, unique_id: Optional[bytes] = None):
        """Seeded random-init weights (see ``weights.random_state_dict``); every
        tensor-parallel rank draws the same full set and keeps its shard."""
        state = random_state_dict(cfg, seed, device=init_device)
        return cls(None, device, cfg=cfg, state=state, tp_rank=tp_rank, tp_size=tp_size, unique_id=unique_id)

    def __del__(self):
        ctx = getattr(self, "ctx", None)
        if ctx is not None and ctx.value:
            try:
                _lib.load().qb_destroy(ctx)
            except Exception:
                pass
            self.ctx = None

    def new_state(self, prompt_length: int, output_length: int, **kw) -> DecodeState:
        self.state = None
        self.state = DecodeState(self, prompt_length, output_length, **kw)
        return self.state

    def generate(self, input_ids: List[List[int]], max_new_tokens: int, draft_tokens: Optional[int] = None,
                 drafter=None):
        """Greedy continuation; yields one token per sequence exactly
        ``max_new_tokens`` times (``dryft/engine/engine.py:202-249``).

        As in the reference, one sequence speculates by default: a
        ``PromptLookup`` over the prompt and the emitted tokens proposes
        ``draft_width(max_new_tokens)`` tokens (up to 7; at most 5 when the
        model has 4 query heads per KV head, so that the verify pass stays on
        the rows attention kernel: ``fast_verify_drafts``), one verify pass
        checks them, and the accepted prefix plus one target token is emitted;
        without a proposal it takes a plain decode step. The emitted sequence
        is the plain greedy one (verification only accepts tokens the target
        itself predicts). ``draft_tokens`` overrides the width (0: plain decode
        with replays running ahead of the consumer); ``drafter`` may be any
        object with ``propose() -> list | None`` and ``append(token)``.

        Several sequences of equal prompt length decode together (every weight
        streamed once per step for up to 8 of them); more than 8 run as chunks
        of 8, each on its own context over the same weights."""
        if max_new_tokens <= 0:
            return
        B = len(input_ids)
        if B < 1:
            raise ValueError("generate needs at least one sequence")
        prompts = [list(p) for p in input_ids]
        if any(len(p) != len(prompts[0]) for p in prompts):
            raise ValueError("the sequences of a batch must have equal prompt lengths")
        if not prompts[0]:
            raise ValueError("the prompt must hold at least one token")
        if draft_tokens is None:
            from .speculate import draft_width, fast_verify_drafts

            width = min(draft_width(max_new_tokens), fast_verify_drafts(self.cfg.n_heads, self.cfg.n_kv_heads))
            draft_tokens = width if B == 1 else 0
        if draft_tokens > 0:
            yield from self._generate_speculative(prompts, max_new_tokens, draft_tokens, drafter)
            return
        if B > DecodeState.MAX_BATCH:
            yield from self._generate_chunked(prompts, max_new_tokens)
            return
        P = len(prompts[0])
        with torch.inference_mode():
            shape = (B, P, max_new_tokens)
            if self.state is None or self.state.shape != shape or self._bound_state is not self.state:
                self.new_state(P, max_new_tokens, batch=B)
            state = self.state
            ids = torch.tensor(prompts if B > 1 else prompts[0], dtype=torch.int64).pin_memory()
            state.prefill(ids.to(self.device, non_blocking=True))
            first = state.read_token()
            yield from stream_decode(state, first, max_new_tokens, depth=self.STREAM_DEPTH)

    def _lane(self, i: int) -> "_Lane":
        """Context i (>= 1) for chunk i of a large batch: its own qb context and
        decode state, borrowing this engine's weights."""
        while len(self._lanes) < i:
            self._lanes.append(_Lane(self))
        return self._lanes[i - 1]

    def _generate_chunked(self, prompts: List[List[int]], max_new_tokens: int):
        """More than 8 sequences: chunks of 8 (the last may be smaller), chunk 0
        on this engine and chunk i on lane i; every step replays each chunk's
        graph, then yields all tokens in sequence order."""
        if self.tp_size > 1:
            raise ValueError("batched decode runs on one GPU")
        M = DecodeState.MAX_BATCH
        chunks = [prompts[i:i + M] for i in range(0, len(prompts), M)]
        P = len(prompts[0])
        with torch.inference_mode():
            states = []
            for i, chunk in enumerate(chunks):
                owner = self if i == 0 else self._lane(i)
                shape = (len(chunk), P, max_new_tokens)
                st = owner.state
                if st is None or st.shape != shape or owner._bound_state is not st:
                    st = owner.new_state(P, max_new_tokens, batch=len(chunk))
                ids = torch.tensor(chunk if len(chunk) > 1 else chunk[0], dtype=torch.int64).pin_memory()
                st.prefill(ids.to(self.device, non_blocking=True))
                states.append(st)
            tokens = [t for st in states for t in st.read_token()]
            for step in range(max_new_tokens):
                if step + 1 < max_new_tokens:
                    for st in states:
                        st.step()
                yield tokens
                if step + 1 < max_new_tokens:
                    tokens = [t for st in states for t in st.read_token()]

    def _generate_speculative(self, input_ids, max_new_tokens: int, k: int, drafter):
        from .speculate import PromptLookup

        if len(input_ids) != 1:
            raise ValueError("speculative decoding takes one sequence")
        prompt = list(input_ids[0])
        if not prompt:
            raise ValueError("the prompt must hold at least one token")
        if not 1 <= k <= 7:
            raise ValueError("draft_tokens must lie in 1..7")
        with torch.inference_mode():
            # capacity holds the draft scratch slots (dryft/engine/decode.py:102-118);
            # the state is shape-keyed like the plain path's (engine.py:212-215)
            shape = (1, len(prompt), max_new_tokens)
            state = self.state
            if (state is None or state.shape != shape or self._bound_state is not state
                    or getattr(state, "draft_tokens", 0) != k):
                state = self.new_state(len(prompt), max_new_tokens, draft_tokens=k)
            ids = torch.tensor(prompt, dtype=torch.int64).pin_memory()
            state.prefill(ids.to(self.device, non_blocking=True))
            tokens = state.read_token()
            yield tokens
            lookup = drafter if drafter is not None else PromptLookup(prompt, draft_length=k)
            lookup.append(tokens[0])
            emitted = 1
            while emitted < max_new_tokens:
                proposal = lookup.propose()
                if proposal:
                    verified = state.verify(tokens[0], list(proposal)[:k])
                    for token in verified[:max_new_tokens - emitted]:
                        tokens = [token]
                        lookup.append(token)
                        emitted += 1
                        yield tokens
                else:
                    state.step()
                    tokens = state.read_token()
                    lookup.append(tokens[0])
                    emitted += 1
                    yield tokens


class _Lane:
    """A second qb context over an engine's weights (no copy), with its own
    decode state: one chunk of a batch larger than 8 sequences. Offers the
    attributes ``DecodeState`` uses from an engine."""

    def __init__(self, engine: Engine):
        self.cfg, self.device, self.tp_size, self.tp_rank = engine.cfg, engine.device, 1, 0
        self.weights = engine.weights
        L = _lib.load()
        cfg = self.cfg
        qc = _lib.QbConfig(cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn, cfg.n_layers,
                           cfg.vocab, cfg.rms_eps)
        ctx = _lib.c_void_p()
        _lib.check(L.qb_create(_lib.ctypes.byref(qc), self.device.index or 0, 0, 1, _lib.ctypes.byref(ctx)))
        self.ctx = ctx
        w = engine.weights
        _lib.check(L.qb_bind_weights(ctx, engine._weight_table, cfg.n_layers, w.embed.data_ptr(),
                                     w.final_norm.data_ptr(), w.lm_head.data_ptr()), ctx)
        self.state: Optional[DecodeState] = None
        self._bound_state = None

    def new_state(self, prompt_length: int, output_length: int, **kw) -> DecodeState:
        self.state = None
        self.state = DecodeState(self, prompt_length, output_length, **kw)
        return self.state

    def __del__(self):
        ctx = getattr(self, "ctx", None)
        if ctx is not None and ctx.value:
            try:
                _lib.load().qb_destroy(ctx)
            except Exception:
                pass
            self.ctx = None
