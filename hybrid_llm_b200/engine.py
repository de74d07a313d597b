"""The reference engine's API (llmy_cuda/include/llmy.h) over this build.

Same names, argument meanings and error behaviour as the engine's C ABI, so a
caller of the reference engine switches by changing the import:

    llmy_load(path) -> model | None          llmy.h:31 / llmy.cpp:21-29
    llmy_free(model)                         llmy.h:32
    llmy_vocab_size / llmy_d_model / llmy_num_loops / llmy_max_loops /
    llmy_mhc_streams / llmy_set_num_loops / llmy_set_fixed_loops
                                             llmy.h:35-41 / llmy.cpp:38-78
    llmy_state_new(model) -> state | None    llmy.h:44 / llmy.cpp:80-89 (batch 1)
    llmy_state_free / llmy_state_reset       llmy.h:45-46 / llmy.cpp:91-114
    llmy_prefill(model, state, tokens, n_tokens, logits_out)
                                             llmy.h:51-53 / model.cpp:1955-1966
    llmy_decode(model, state, token, position, num_loops, logits_out)
                                             llmy.h:57-59 / model.cpp:1968-1972
    llmy_sample(logits, vocab_size, temperature, top_k, top_p,
                repetition_penalty, recent_tokens, n_recent, rng_state)
                                             llmy.h:64-68 / llmy.cpp:132-202
    llmy_last_executed_loops(state), llmy_sync()
                                             llmy.h:71-72
    llmy_mhc_sinkhorn4, llmy_moe_selected_fp32
                                             llmy.h:74-88 (device buffers, int status)

A model is the checkpoint in the engine's ``.llmy`` format loaded onto one GPU
(``ModelWeights.from_llmy``) and served by LoopedHybridModel: prefill runs the
whole prompt through the batched kernels (the reference steps token by token,
model.cpp:1958-1965, with the same result up to rounding), decode runs one
step at the given position.  ``logits_out`` is any writable float32 buffer of
vocab_size elements: a numpy array, a host or CUDA torch tensor, or a ctypes
array.  ``llmy_sample`` runs on the host, as in the reference, through the
native library (llmyb_engine_sample).  Load and state-creation failures print
``[llmy_load] ...`` / ``[llmy_state_new] ...`` to stderr and return None.
"""
from __future__ import annotations

import ctypes
import dataclasses
import sys
from pathlib import Path

import numpy as np
import torch

from . import _native
from .config import HybridConfig
from .model import LoopedHybridModel
from .state import RecurrentState
from .weights import ModelWeights


class LlmyModel:
    """Handle returned by llmy_load (the reference's opaque llmy_model)."""

    def __init__(self, model: LoopedHybridModel, path: Path):
        self.model = model
        self.cfg: HybridConfig = model.cfg
        self.path = path
        self.num_loops = int(self.cfg.num_loops)


class LlmyState:
    """Handle returned by llmy_state_new: one sequence's recurrent state."""

    def __init__(self, m: LlmyModel):
        self.cfg = dataclasses.replace(m.cfg, num_loops=max(m.cfg.num_loops, m.num_loops))
        self.state = RecurrentState(self.cfg, 1, m.model.device)
        self.position = 0
        self.last_executed_loops = 0


# ------------------------------------------------------------- model lifecycle
def llmy_load(path: str | bytes | Path, device: str | torch.device = "cuda") -> LlmyModel | None:
    """Load a ``.llmy`` checkpoint onto `device`; None (and a message on
    stderr) if the file cannot be read or describes an unsupported model."""
    try:
        p = Path(path.decode() if isinstance(path, bytes) else path)
        return LlmyModel(LoopedHybridModel(ModelWeights.from_llmy(p, device)), p)
    except Exception as exc:  # the reference reports any failure this way
        print(f"[llmy_load] {exc}", file=sys.stderr)
        return None


def llmy_free(m: LlmyModel | None) -> None:
    """Release the model's device memory (a None handle is ignored)."""
    if m is None:
        return
    m.model = None


def _live(m: LlmyModel) -> LoopedHybridModel:
    if m is None or m.model is None:
        raise ValueError("model handle is null or freed")
    return m.model


# --------------------------------------------------------------- introspection
def llmy_vocab_size(m: LlmyModel) -> int:
    return int(m.cfg.vocab_size)


def llmy_d_model(m: LlmyModel) -> int:
    return int(m.cfg.d_model)


def llmy_num_loops(m: LlmyModel) -> int:
    return int(m.num_loops)


def llmy_max_loops(m: LlmyModel) -> int:
    """Adaptive halting is not part of the served models, so the maximum is
    the configured loop count (llmy.cpp:53-59 without adaptive_max_loops)."""
    return int(m.num_loops)


def llmy_mhc_streams(m: LlmyModel) -> int:
    """Residual streams: 1 (multi-stream hyper-connections are rejected at load)."""
    return 1


def llmy_set_num_loops(m: LlmyModel, n: int) -> None:
    """Default loop count of prefill and decode, and decode's upper bound.
    States created afterwards hold state for that many loops."""
    n = int(n)
    if n < 1:
        raise ValueError(f"num_loops must be >= 1, got {n}")
    m.num_loops = n


def llmy_set_fixed_loops(m: LlmyModel, n: int) -> None:
    """Fix the loop count (n < 1 is ignored, as in the reference)."""
    if int(n) >= 1:
        m.num_loops = int(n)


# -------------------------------------------------------------- state lifecycle
def llmy_state_new(m: LlmyModel) -> LlmyState | None:
    try:
        _live(m)
        return LlmyState(m)
    except Exception as exc:
        print(f"[llmy_state_new] {exc}", file=sys.stderr)
        return None


def llmy_state_free(s: LlmyState | None) -> None:
    if s is not None:
        s.state = None


def llmy_state_reset(s: LlmyState | None) -> None:
    """Zero every state tensor (a fresh conversation)."""
    if s is None:
        return
    s.state.zero_()
    s.position = 0
    s.last_executed_loops = 0


# ------------------------------------------------------------------- forwards
def _token_tensor(tokens, n_tokens: int, device) -> torch.Tensor:
    if isinstance(tokens, torch.Tensor):
        t = tokens.reshape(-1)[:n_tokens]
    else:
        if isinstance(tokens, ctypes.Array):
            tokens = np.ctypeslib.as_array(tokens)
        t = torch.as_tensor(np.asarray(tokens).reshape(-1)[:n_tokens])
    if t.numel() != n_tokens:
        raise ValueError(f"tokens holds {t.numel()} ids, n_tokens is {n_tokens}")
    return t.to(device=device, dtype=torch.int64).reshape(1, n_tokens)


def _write_logits(logits_out, row: torch.Tensor) -> None:
    """Copy one fp32 logits row into the caller's buffer (host or device)."""
    row = row.reshape(-1).float()
    if isinstance(logits_out, torch.Tensor):
        if (logits_out.dtype != torch.float32 or logits_out.numel() < row.numel()
                or not logits_out.is_contiguous()):
            raise ValueError("logits_out must be a contiguous buffer of vocab_size float32 values")
        logits_out.reshape(-1)[:row.numel()].copy_(row)
        return
    if isinstance(logits_out, ctypes.Array):
        logits_out = np.ctypeslib.as_array(logits_out)
    out = np.asarray(logits_out)
    if out.dtype != np.float32 or out.size < row.numel() or not out.flags.c_contiguous:
        raise ValueError("logits_out must be a contiguous buffer of vocab_size float32 values")
    out.reshape(-1)[:row.numel()] = row.cpu().numpy()


def _check_loops(s: LlmyState, loops: int) -> None:
    if s is None or s.state is None:
        raise ValueError("state handle is null or freed")
    if loops > s.cfg.num_loops:
        raise ValueError(f"the state holds {s.cfg.num_loops} loops, {loops} requested "
                         "(create the state after llmy_set_num_loops)")


def llmy_prefill(m: LlmyModel, s: LlmyState, tokens, n_tokens: int, logits_out) -> None:
    """Run the prompt tokens[0:n_tokens] at positions 0..n_tokens-1 and write
    the last token's logits; n_tokens <= 0 does nothing."""
    model = _live(m)
    _check_loops(s, m.num_loops)
    n_tokens = int(n_tokens)
    if n_tokens <= 0:
        return
    ids = _token_tensor(tokens, n_tokens, model.device)
    out = model.forward(ids, state=s.state, last_logits_only=True, num_loops=m.num_loops)
    _write_logits(logits_out, out.logits[0, -1])
    s.position = n_tokens - 1
    s.last_executed_loops = m.num_loops


def llmy_decode(m: LlmyModel, s: LlmyState, token: int, position: int, num_loops: int,
                logits_out) -> None:
    """One step for `token` at absolute position `position`; num_loops 0 (or
    negative) means the model default, larger values are capped at it."""
    model = _live(m)
    loops = int(num_loops) if int(num_loops) > 0 else m.num_loops
    loops = min(loops, m.num_loops)
    _check_loops(s, loops)
    s.state.positions.fill_(int(position))
    ids = torch.tensor([int(token)], dtype=torch.int64, device=model.device)
    logits = model.decode_step(ids, s.state, num_loops=loops)
    _write_logits(logits_out, logits[0])
    s.position = int(position)
    s.last_executed_loops = loops


# ------------------------------------------------------------------- sampling
def llmy_sample(logits, vocab_size: int, temperature: float, top_k: int, top_p: float,
                repetition_penalty: float, recent_tokens, n_recent: int, rng_state) -> int:
    """The engine's host sampler.  logits: host float32 [vocab_size] (numpy,
    CPU torch tensor or ctypes array; a CUDA tensor is copied to the host);
    recent_tokens: int32 ids (or None); rng_state: a ctypes.c_uint64 or a
    uint64 numpy array, advanced in place.  Returns the token id."""
    if isinstance(logits, torch.Tensor):
        logits = logits.detach().reshape(-1).float().cpu().numpy()
    elif isinstance(logits, ctypes.Array):
        logits = np.ctypeslib.as_array(logits)
    lg = np.ascontiguousarray(np.asarray(logits, dtype=np.float32).reshape(-1))
    vocab_size = int(vocab_size)
    if vocab_size > lg.size:
        raise ValueError(f"logits holds {lg.size} values, vocab_size is {vocab_size}")
    n_recent = int(n_recent) if recent_tokens is not None else 0
    rec = None
    if n_recent > 0:
        rec = np.ascontiguousarray(np.asarray(recent_tokens, dtype=np.int32).reshape(-1)[:n_recent])
        if rec.size != n_recent:
            raise ValueError(f"recent_tokens holds {rec.size} ids, n_recent is {n_recent}")
    if isinstance(rng_state, ctypes.c_uint64):
        holder, arr = rng_state, None
    else:
        arr = rng_state
        if not (isinstance(arr, np.ndarray) and arr.dtype == np.uint64 and arr.size >= 1):
            raise TypeError("rng_state must be a ctypes.c_uint64 or a uint64 numpy array")
        holder = ctypes.c_uint64(int(arr.reshape(-1)[0]))
    tok = _native.lib().llmyb_engine_sample(
        lg.ctypes.data, vocab_size, float(temperature), int(top_k), float(top_p),
        float(repetition_penalty), None if rec is None else rec.ctypes.data, n_recent,
        ctypes.byref(holder))
    if tok < 0:
        raise ValueError("llmy_sample: invalid arguments")
    if arr is not None:
        arr.reshape(-1)[0] = holder.value
    return int(tok)


# ------------------------------------------------------- device entry points
def _addr(p) -> int | None:
    if p is None:
        return None
    if isinstance(p, torch.Tensor):
        if not p.is_cuda:
            raise ValueError("device pointers only: pass CUDA tensors or raw addresses")
        return p.data_ptr()
    return int(p)


def _stream_handle(stream) -> int | None:
    if stream is None:
        return None
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


def llmy_mhc_sinkhorn4(input, output, matrices: int, iterations: int, stream=None) -> int:
    """Sinkhorn normalisation of fp32 [matrices, 4, 4] device data (CUDA tensors
    or raw addresses); returns the status (0 = success, 1 = invalid value)."""
    return int(_native.lib().llmyb_mhc_sinkhorn4(_addr(input), _addr(output), int(matrices),
                                                  int(iterations), _stream_handle(stream)))


def llmy_moe_selected_fp32(x, idx, prob, gate_up, down, activation, route_output, out,
                           D: int, H: int, E: int, k: int, stream=None) -> int:
    """One token through its k routed experts, fp32, on device buffers (CUDA
    tensors or raw addresses); returns the status (0 = success)."""
    return int(_native.lib().llmyb_moe_selected_fp32(
        *(_addr(t) for t in (x, idx, prob, gate_up, down, activation, route_output, out)),
        int(D), int(H), int(E), int(k), _stream_handle(stream)))


# ---------------------------------------------------------------- diagnostics
def llmy_last_executed_loops(s: LlmyState) -> int:
    return int(s.last_executed_loops)


def llmy_sync() -> None:
    torch.cuda.synchronize()
