"""Greedy generation over the per-rank KV cache (reference: minitp/generation.py).

``GenerationState`` keeps the reference API (prefill / select_next / append /
decode_step, ``out_ids``, ``positions_buf``, ``cursor``). ``generate_greedy``
(distributed argmax, up to 64 rows) runs the decode loop as replays of one
CUDA graph; with an EOS id and ``early_stop`` it checks on the host after
each replay whether every row finished, as the reference loop does. The graph holds one captured
``mtpb_model_decode_step``: the embedding of the current token, all layers,
the LM head with the packed-key argmax, the NVLink exchange of the winners,
and the write of the token to ``out_ids[:, pos + 1]`` with the position
advance. Token, position and collective sequence numbers live on the
device, so replays need no host input and no synchronisation.
"""

from __future__ import annotations

import torch

from minitp_b200 import _lib, ops
from minitp_b200.distributed import all_gather
from minitp_b200.kv_cache import KVCache
from minitp_b200.layer import TPQwen2ForCausalLM


def _kv_heads_local(model: TPQwen2ForCausalLM) -> int:
    return model.model.layers[0].self_attn.kv_heads_local


def make_kv_cache(model: TPQwen2ForCausalLM, batch_size: int, max_seq_len: int, init: str = "empty") -> KVCache:
    """Reference: generation.py:36-51."""
    p = next(model.parameters())
    return KVCache(model.cfg.num_hidden_layers, batch_size, _kv_heads_local(model), model.cfg.head_dim,
                   max_seq_len, p.dtype, p.device, init=init)


def select_token(model: TPQwen2ForCausalLM, logits: torch.Tensor, distributed_argmax: bool = True) -> torch.Tensor:
    """Greedy pick from local logits ``[B, T, V_local]``; identical on every rank (generation.py:54-67)."""
    if distributed_argmax:
        return model.lm_head.distributed_argmax(logits[:, -1]).squeeze(-1)
    if model.ctx.tp_size == 1:
        return ops.argmax(logits[:, -1], 0, None).squeeze(-1)
    full = torch.empty(*logits.shape[:-2], model.cfg.vocab_size, dtype=logits.dtype, device=logits.device)
    all_gather(full, logits[:, -1].contiguous(), model.ctx.process_group)
    return ops.argmax(full, 0, None).squeeze(-1)


class DecodeSession:
    """Buffers of one (batch, total length) shape kept on the model between
    ``generate_greedy`` calls: the KV cache, the output ids, the positions,
    the device token, and the CUDA graph of the decode step captured over
    them. A later call of the same shape replays that graph instead of
    running an eager step and capturing a new graph (a few ms per call).
    Sessions are dropped whenever the model's native handle is released.
    """

    def __init__(self, model: TPQwen2ForCausalLM, batch: int, total: int, device: torch.device, native: int) -> None:
        self.kv = make_kv_cache(model, batch, total)
        self.out_ids = torch.empty(batch, total, dtype=torch.long, device=device)
        self.positions = torch.arange(total, device=device)
        self.tok = torch.empty(batch, dtype=torch.int64, device=device)
        self.graph: torch.cuda.CUDAGraph | None = None
        self.graph_epoch = -1  # library settings epoch at the graph's capture
        self.native = native  # handle of the native model the graph runs

    def usable_graph(self) -> torch.cuda.CUDAGraph | None:
        """The captured graph, unless a library setting changed since its capture."""
        if self.graph is not None and self.graph_epoch != _lib.load().mtpb_settings_epoch():
            self.graph = None
        return self.graph


_MAX_SESSIONS = 4


def decode_session(model: TPQwen2ForCausalLM, batch: int, total: int, device: torch.device) -> DecodeSession:
    """The model's session for this shape (created on first use; at most four kept)."""
    native = model.native()  # first: (re)building the native model drops the model's sessions
    cache = model.__dict__.setdefault("_decode_sessions", {})
    key = (batch, total, str(device))
    s = cache.pop(key, None)
    if s is None or s.native != native:
        s = DecodeSession(model, batch, total, device, native)
    cache[key] = s  # most recently used last
    while len(cache) > _MAX_SESSIONS:
        cache.pop(next(iter(cache)))
    return s


class GenerationState:
    """KV cache + positions buffer + output buffer (reference generation.py:70-130)."""

    def __init__(
        self,
        model: TPQwen2ForCausalLM,
        input_ids: torch.Tensor,
        max_new_tokens: int,
        kv: KVCache | None = None,
        distributed_argmax: bool = True,
        kv_init: str = "empty",
        session: DecodeSession | None = None,
    ) -> None:
        self.model = model
        self.distributed_argmax = distributed_argmax
        b, t = input_ids.shape
        self.batch = b
        self.prompt_len = t
        self.max_new_tokens = max_new_tokens
        self.total = t + max_new_tokens
        device = input_ids.device
        self._session = session
        if session is not None:
            self.kv = session.kv
            self.kv.seq_len = 0
            self.out_ids = session.out_ids
            self.positions_buf = session.positions
        else:
            self.kv = kv if kv is not None else make_kv_cache(model, b, self.total, init=kv_init)
            self.out_ids = torch.empty(b, self.total, dtype=torch.long, device=device)
            self.positions_buf = torch.arange(self.total, device=device)
        self.out_ids[:, :t] = input_ids
        self.cursor = t
        self.finished: torch.Tensor | None = None
        self.eos = -1
        self._graph: torch.cuda.CUDAGraph | None = None
        self._tok: torch.Tensor | None = None

    def prefill(self, last_only: bool = False) -> torch.Tensor:
        positions = self.positions_buf[: self.prompt_len]
        return self.model(self.out_ids[:, : self.prompt_len], positions=positions, kv_cache=self.kv,
                          last_only=last_only)

    def select_next(self, logits: torch.Tensor) -> torch.Tensor:
        return select_token(self.model, logits, self.distributed_argmax)

    def append(self, tok: torch.Tensor) -> torch.Tensor:
        self.out_ids[:, self.cursor] = tok
        pos = self.positions_buf[self.cursor]
        self.cursor += 1
        return pos

    def decode_step(self, tok: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        return self.model(tok.unsqueeze(-1), positions=pos.unsqueeze(-1), kv_cache=self.kv)

    # ------------------------------------------------------------------
    # device-resident decode (graph replays)
    # ------------------------------------------------------------------
    def _step_args(self):
        kp, vp = self.kv.pointer_arrays()
        return (self.model.native(), self._tok.data_ptr(), self.batch, kp, vp, self.kv.max_seq_len,
                self.out_ids.data_ptr(), self.total, None)

    def start_device_decode(self, tok: torch.Tensor) -> None:
        """Seed the device loop with the token just appended at ``cursor - 1``."""
        if self.batch > 64:
            raise ValueError("device decode supports at most 64 rows")
        comm = self.model.ctx.comm()
        if self._session is not None:
            self._tok = self._session.tok
            self._tok.copy_(tok.to(torch.int64))
            self._graph = self._session.usable_graph()
        else:
            self._tok = tok.to(torch.int64).contiguous().clone()
        _lib.call("mtpb_comm_set_pos", comm.handle, self.cursor - 1, _lib.stream_ptr(self._tok.device))
        h = self.model.native()
        _lib.call("mtpb_model_reserve", h, self.batch, self.kv.max_seq_len)

    def device_step(self) -> None:
        """One decode step + greedy selection, all on the device (no graph)."""
        self.kv.check_room(1)
        _lib.call("mtpb_model_decode_step", *self._step_args(), _lib.stream_ptr(self._tok.device))
        self.kv.advance(1)
        self.cursor += 1

    def capture(self) -> None:
        """Capture one device decode step into a CUDA graph."""
        g = torch.cuda.CUDAGraph()
        args = self._step_args()
        with torch.cuda.graph(g):
            _lib.call("mtpb_model_decode_step", *args, _lib.stream_ptr(self._tok.device))
        self._graph = g
        if self._session is not None:
            self._session.graph = g
            self._session.graph_epoch = _lib.load().mtpb_settings_epoch()

    def graph_step(self) -> None:
        self.kv.check_room(1)
        self._graph.replay()
        self.kv.advance(1)
        self.cursor += 1

    def run_fixed(self, use_graph: bool = True) -> torch.Tensor:
        """Fixed-length greedy generation (the reference loop with early_stop=False)."""
        logits = self.prefill(last_only=True)
        tok = self.select_next(logits)
        self.append(tok)
        steps = self.max_new_tokens - 1
        if steps <= 0:
            return self.out_ids
        self.start_device_decode(tok)
        if use_graph and self._graph is not None:  # a session's graph of this shape
            for _ in range(steps):
                self.graph_step()
            return self.out_ids
        self.device_step()  # first step eagerly: sets function attributes, validates the chain
        if steps > 1:
            if use_graph:
                self.capture()
                for _ in range(steps - 1):
                    self.graph_step()
            else:
                for _ in range(steps - 1):
                    self.device_step()
        return self.out_ids

    def run_until_eos(self, eos_token_id: int, use_graph: bool = True) -> torch.Tensor:
        """Greedy generation that stops once every row emitted EOS.

        The reference loop (generation.py:147-171): a finished row keeps
        emitting EOS and the loop ends at the first step where all rows are
        finished (one host check per step, as there). The steps themselves are
        the same device decode steps as ``run_fixed``, so both loops produce
        the same ids up to the stop.
        """
        dev = self.out_ids.device
        self.eos = eos_token_id
        self.finished = torch.zeros(self.batch, dtype=torch.bool, device=dev)
        eos_t = torch.tensor(eos_token_id, dtype=torch.long, device=dev)
        tok = self.select_next(self.prefill(last_only=True))
        for step in range(self.max_new_tokens):
            if step > 0:
                if self._graph is not None:
                    self.graph_step()
                else:
                    self.device_step()
                    if use_graph and step + 1 < self.max_new_tokens:
                        self.capture()
                tok = self._tok
            tok = torch.where(self.finished, eos_t, tok)
            self.finished |= tok == eos_token_id
            if step == 0:
                self.append(tok)
            else:
                self.out_ids[:, self.cursor - 1] = tok
                self._tok.copy_(tok)
            if bool(self.finished.all()):
                break
            if step == 0 and self.max_new_tokens > 1:
                self.start_device_decode(tok)
        return self.out_ids[:, : self.cursor]

    def release(self) -> None:
        self._graph = None


@torch.inference_mode()
def generate_greedy(
    model: TPQwen2ForCausalLM,
    input_ids: torch.Tensor,
    max_new_tokens: int,
    eos_token_id: int | None = None,
    distributed_argmax: bool = True,
    early_stop: bool = True,
    kv: KVCache | None = None,
    kv_init: str = "empty",
) -> torch.Tensor:
    """Greedy decode (reference generation.py:133-171).

    Returns ``[B, prompt + generated]``: trimmed at the first step where all
    rows hit EOS when ``early_stop=True``; exactly prompt + max_new_tokens
    columns otherwise.
    """
    b = input_ids.shape[0]
    fixed = not (early_stop and eos_token_id is not None)
    if distributed_argmax and b <= 64:
        # device decode loop: replays of one captured step, buffers kept per shape
        session = None
        if kv is None and kv_init == "empty":
            session = decode_session(model, b, input_ids.shape[1] + max_new_tokens, input_ids.device)
        state = GenerationState(model, input_ids, max_new_tokens, kv=kv, distributed_argmax=distributed_argmax,
                                kv_init=kv_init, session=session)
        if fixed:
            out = state.run_fixed(use_graph=True)
            out = out if not early_stop else out[:, : state.cursor]
        else:
            out = state.run_until_eos(eos_token_id, use_graph=True)
        state.release()
        return out.clone() if session is not None else out
    state = GenerationState(model, input_ids, max_new_tokens, kv=kv, distributed_argmax=distributed_argmax,
                            kv_init=kv_init)
    if early_stop and eos_token_id is not None:
        state.eos = eos_token_id
        state.finished = torch.zeros(b, dtype=torch.bool, device=input_ids.device)
    logits = state.prefill(last_only=True)
    eos_tok = torch.tensor(state.eos, device=input_ids.device)
    for step in range(max_new_tokens):
        tok = state.select_next(logits)
        if state.finished is not None:
            tok = torch.where(state.finished, eos_tok, tok)
            state.finished = state.finished | (tok == state.eos)
        pos = state.append(tok)
        if state.finished is not None and bool(state.finished.all()):
            break
        if step + 1 < max_new_tokens:
            logits = state.decode_step(tok, pos)
    return state.out_ids[:, : state.cursor] if early_stop else state.out_ids


__all__ = ["DecodeSession", "GenerationState", "decode_session", "generate_greedy", "make_kv_cache", "select_token"]
