"""Continuous batching of generation requests over a LlamaModel's KV slots
(csrc/sched.cpp through the C ABI).

The reference's server answers one request at a time: the prompt through
forwardStep, then Sampler.sample -> forwardStep per token with the prompt
plus the emitted tokens as the repetition-penalty history, stopping at
maxTokens or the EOS id (server/InferenceServer.java:111-134). Here each
request owns a KV slot while it runs and every step() advances all of them
with one batched decode step and device sampling.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import call
from .inference import LlamaModel, SamplerConfig, _sampler_array


class BatchScheduler:
    def __init__(self, model: LlamaModel):
        self.model = model
        self._h = C.c_void_p()
        call("at_sched_create", model._h, C.byref(self._h))

    def submit(self, promptTokenIds, maxTokens: int, config: SamplerConfig, eosTokenId: int = -1) -> int:
        """Queues a request; returns its id."""
        p = np.ascontiguousarray(np.asarray(promptTokenIds, dtype=np.int32))
        cfg, keep = _sampler_array([config], None)
        rid = C.c_int()
        call("at_sched_submit", self._h, p.ctypes.data_as(C.c_void_p), int(p.size), int(maxTokens), int(eosTokenId),
             C.cast(cfg, C.c_void_p), C.byref(rid))
        del keep
        return rid.value

    def step(self) -> int:
        """Admits waiting requests, runs one batched step; returns the number of
        requests still running or waiting."""
        n = C.c_int()
        call("at_sched_step", self._h, C.byref(n))
        return n.value

    def result(self, requestId: int) -> tuple[np.ndarray, bool]:
        """The tokens generated so far and whether the request is finished."""
        n, done = C.c_int(), C.c_int()
        call("at_sched_result", self._h, int(requestId), None, 0, C.byref(n), C.byref(done))
        out = np.empty(max(1, n.value), dtype=np.int32)
        call("at_sched_result", self._h, int(requestId), out.ctypes.data_as(C.c_void_p), n.value, C.byref(n),
             C.byref(done))
        return out[: n.value], bool(done.value)

    def runToCompletion(self, max_steps: int = 1 << 30) -> int:
        """Steps until no request is left; returns the number of steps."""
        steps = 0
        while steps < max_steps:
            steps += 1
            if self.step() == 0:
                break
        return steps

    def close(self) -> None:
        if self._h:
            call("at_sched_destroy", self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
