"""Byte generation with the mini transformer on the GPU.

Mirrors generate_mini_transformer (crates/nsrl-train/src/lib.rs:12702-12800)
for base-2 softmax attention, batched over sequences: every step runs the
full forward of each context's last seq_len bytes (left-padded with ' '),
the byte head on the last position and the choice of the next byte, all on
the device (nsrl_mini_transformer_generate); the host reads the tokens once
at the end.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence

import torch

from . import core
from . import train as T

STRATEGIES = {"greedy": 0, "sample": 1}


class DecodeConfigC(C.Structure):
    _fields_ = [("strategy", C.c_int32), ("top_k", C.c_uint32), ("sample_seed", C.c_uint64)]


def _lib():
    L = T._lib_bwd()
    if not getattr(L, "_gen_bound", False):
        vp, sz = C.c_void_p, C.c_size_t
        L.nsrl_generate_workspace_size.restype = sz
        L.nsrl_generate_workspace_size.argtypes = [vp, sz]
        L.nsrl_mini_transformer_output_rows.argtypes = [vp, vp, sz, vp, vp, vp, sz, vp, vp]
        L.nsrl_mini_transformer_generate.argtypes = [vp, vp, sz, vp, sz, sz, C.POINTER(DecodeConfigC), vp, vp, vp,
                                                     vp, sz, vp, vp]
        L._gen_bound = True
    return L


def output_rows(model: T.TrainModel, windows: torch.Tensor):
    """The byte-head row of each window's last position (lib.rs:14911-15008,
    :17455-17490): (logits_q8 int32 [B, 256], probs_q15 int16 [B, 256]), or
    None when a window is rejected."""
    L = _lib()
    w = windows.to(core._dev(), torch.uint8).contiguous()
    B = w.shape[0]
    m = model.c()
    logits = torch.empty((B, 256), dtype=torch.int32, device=w.device)
    probs = torch.empty((B, 256), dtype=torch.int16, device=w.device)
    ws = core.workspace(L.nsrl_generate_workspace_size(C.byref(m), B))
    st = core.Status()
    st.reset()
    r = L.nsrl_mini_transformer_output_rows(C.byref(m), core._ptr(w), B, core._ptr(logits), core._ptr(probs),
                                            core._ptr(ws), ws.numel(), core._ptr(st.buf), core._stream())
    return (logits, probs) if T._run_status(r, st) else None


class Generator:
    """Workspace and context buffers for generating `steps` bytes after
    prompts of up to `max_prompt` bytes, for `batch` sequences at a time."""

    def __init__(self, model: T.TrainModel, batch: int, max_prompt: int, steps: int):
        L = _lib()
        self.model, self.batch, self.steps = model, batch, steps
        self.capacity = max_prompt + steps
        m = model.c()
        nbytes = L.nsrl_generate_workspace_size(C.byref(m), batch)
        if nbytes == 0:
            raise ValueError(L.nsrl_last_error().decode() or "invalid generation shape")
        dev = core._dev()
        self.ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        self.contexts = torch.empty((batch, self.capacity), dtype=torch.uint8, device=dev)
        self.tokens = torch.empty((batch, steps), dtype=torch.uint8, device=dev)
        self.pick_logits = torch.empty((batch, steps), dtype=torch.int32, device=dev)
        self.pick_probs = torch.empty((batch, steps), dtype=torch.int16, device=dev)
        self.status = core.Status()

    def launch(self, prompt_lens: Sequence[int], strategy="greedy", top_k=0, seed=0) -> int:
        """Enqueues a generation over self.contexts (prompts already copied in);
        returns the C status code."""
        L = _lib()
        lens = (C.c_int32 * self.batch)(*[int(n) for n in prompt_lens])
        cfg = DecodeConfigC(STRATEGIES[strategy], int(top_k), int(seed))
        m = self.model.c()
        return L.nsrl_mini_transformer_generate(C.byref(m), core._ptr(self.contexts), self.capacity, lens,
                                                self.batch, self.steps, C.byref(cfg), core._ptr(self.tokens),
                                                core._ptr(self.pick_logits), core._ptr(self.pick_probs),
                                                core._ptr(self.ws), self.ws.numel(), core._ptr(self.status.buf),
                                                core._stream())

    def __call__(self, prompts: Sequence[bytes], strategy="greedy", top_k=0, seed=0):
        """Generates for each prompt; returns (tokens uint8 [B, steps], the
        picks' logits, the picks' probabilities) as host tensors, or None on a
        rejection."""
        if len(prompts) != self.batch:
            raise ValueError("one prompt per sequence of the batch")
        host = torch.zeros((self.batch, self.capacity), dtype=torch.uint8)
        for b, p in enumerate(prompts):
            if len(p) + self.steps > self.capacity:
                raise ValueError("prompt longer than the generator's max_prompt")
            host[b, :len(p)] = torch.frombuffer(bytearray(p), dtype=torch.uint8)
        self.contexts.copy_(host)
        self.status.reset()
        r = self.launch([len(p) for p in prompts], strategy, top_k, seed)
        if not T._run_status(r, self.status):
            return None
        return self.tokens.cpu(), self.pick_logits.cpu(), self.pick_probs.cpu()


class StreamingGenerator:
    """Incremental generation with a one-layer linear-attention model without
    positions (generate_mini_transformer_streaming_linear_nope_with_priors and
    its TTT variant, lib.rs:12802-12980): each stream carries its linear
    attention state; prompts of one length per batch."""

    def __init__(self, model: T.TrainModel, batch: int, prompt_len: int, steps: int):
        L = _lib()
        if not getattr(L, "_sgen_bound", False):
            vp, sz = C.c_void_p, C.c_size_t
            L.nsrl_generate_streaming_workspace_size.restype = sz
            L.nsrl_generate_streaming_workspace_size.argtypes = [vp, sz]
            L.nsrl_mini_transformer_generate_streaming.argtypes = [vp, vp, sz, sz, sz, sz, C.POINTER(DecodeConfigC),
                                                                   C.c_int, vp, vp, vp, vp, sz, vp, vp]
            L._sgen_bound = True
        self.model, self.batch, self.prompt_len, self.steps = model, batch, prompt_len, steps
        self.capacity = prompt_len + steps
        m = model.c()
        nbytes = L.nsrl_generate_streaming_workspace_size(C.byref(m), batch)
        if nbytes == 0:
            raise ValueError(L.nsrl_last_error().decode() or "invalid streaming-generation shape")
        dev = core._dev()
        self.ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        self.contexts = torch.empty((batch, self.capacity), dtype=torch.uint8, device=dev)
        self.tokens = torch.empty((batch, steps), dtype=torch.uint8, device=dev)
        self.pick_logits = torch.empty((batch, steps), dtype=torch.int32, device=dev)
        self.pick_probs = torch.empty((batch, steps), dtype=torch.int16, device=dev)
        self.status = core.Status()

    def __call__(self, prompts: Sequence[bytes], strategy="greedy", top_k=0, seed=0, ttt_shift=None):
        if len(prompts) != self.batch or any(len(p) != self.prompt_len for p in prompts):
            raise ValueError("one prompt of prompt_len bytes per stream")
        L = _lib()
        host = torch.zeros((self.batch, self.capacity), dtype=torch.uint8)
        for b, p in enumerate(prompts):
            host[b, :len(p)] = torch.frombuffer(bytearray(p), dtype=torch.uint8)
        self.contexts.copy_(host)
        self.status.reset()
        cfg = DecodeConfigC(STRATEGIES[strategy], int(top_k), int(seed))
        m = self.model.c()
        r = L.nsrl_mini_transformer_generate_streaming(
            C.byref(m), core._ptr(self.contexts), self.capacity, self.prompt_len, self.batch, self.steps,
            C.byref(cfg), -1 if ttt_shift is None else int(ttt_shift), core._ptr(self.tokens),
            core._ptr(self.pick_logits), core._ptr(self.pick_probs), core._ptr(self.ws), self.ws.numel(),
            core._ptr(self.status.buf), core._stream())
        if not T._run_status(r, self.status):
            return None
        return self.tokens.cpu(), self.pick_logits.cpu(), self.pick_probs.cpu()
