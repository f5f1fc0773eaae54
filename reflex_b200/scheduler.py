"""Asynchronous chunk scheduling: the next action chunk is computed on the GPU
while the robot executes the current one.

* ``ChunkScheduler`` is the control-loop manager of reflex/run.py:47-252
  (AsyncInferenceManager) and reflex/run_streaming.py:104-175:
  - the first chunk is computed synchronously;
  - ``overlap_steps`` actions before the current chunk ends, the next
    inference is launched with future-state substitution: the observation's
    state is replaced by the current chunk's last action (zero-padded or
    truncated to the state's width), the state the robot will be in when the
    new chunk starts;
  - at the chunk boundary the pending chunk becomes the current one.
  On a CUDA policy the launch is asynchronous: the chunk is enqueued on the
  scheduler's own CUDA stream and copied into pinned host memory behind an
  event, so ``get_action`` returns immediately and only the switch waits (if
  the GPU is not done yet).  In streaming mode every inference after the
  first passes ``incremental_input=True`` (run_streaming.py:163-170).
* ``PrefillDecodeStreams`` is ConcurrentStreamingExecutor
  (reflex/policies/pi05/concurrent_executor.py:26-189) with CUDA streams:
  the prefill (frame update) runs on one stream and records an event; the
  decode runs on another and waits for that event only when it needs the
  new context.
"""
from __future__ import annotations

from copy import copy

import numpy as np
import torch


class _Pending:
    """A chunk whose computation has been enqueued: pinned host copy + event."""

    def __init__(self, host: torch.Tensor, event):
        self.host, self.event = host, event

    def result(self) -> np.ndarray:
        if self.event is not None:
            self.event.synchronize()
        return self.host.numpy().copy()


class ChunkScheduler:
    def __init__(self, policy, n_action_steps: int, overlap_steps: int, *, streaming: bool = False,
                 state_key: str = "observation.state"):
        if n_action_steps < overlap_steps:
            raise ValueError("n_action_steps must be greater than or equal to overlap_steps")
        if overlap_steps < 0:
            raise ValueError("overlap_steps must be non-negative")
        self.policy = policy
        self.n_action_steps, self.overlap_steps = n_action_steps, overlap_steps
        self.streaming = streaming
        self.state_key = state_key
        self.current_chunk: np.ndarray | None = None  # executing, on the host
        self.next_chunk: _Pending | None = None  # enqueued on the GPU
        self.chunk_index = 0
        self._incremental = False
        self.launches: list[dict] = []  # (chunk_index, state used) of every inference, for inspection
        self.stream = None

    # ------------------------------------------------------------ state ---
    def is_running(self) -> bool:
        return self.current_chunk is not None or self.next_chunk is not None

    def should_switch_chunk(self) -> bool:
        return self.chunk_index == 0

    def should_launch_next_inference(self) -> bool:
        return self.chunk_index == self.n_action_steps - self.overlap_steps

    def should_fetch_observation(self) -> bool:
        return not self.is_running() or self.should_launch_next_inference()

    def get_current_action(self) -> np.ndarray:
        if self.current_chunk is None:
            raise RuntimeError("No chunk is currently executing")
        return self.current_chunk[self.chunk_index]

    # -------------------------------------------------------- inference ---
    def _future_state(self, observation: dict) -> dict:
        observation = copy(observation)
        if self.current_chunk is not None and self.state_key in observation:
            last = np.asarray(self.current_chunk[self.n_action_steps - 1])
            state = observation[self.state_key]
            dim = state.shape[-1]
            if isinstance(state, torch.Tensor):
                new = torch.zeros_like(state)
                n = min(dim, last.shape[-1])
                new[..., :n] = torch.as_tensor(last[..., :n], dtype=state.dtype, device=state.device)
            else:
                new = np.zeros_like(state)
                n = min(dim, last.shape[-1])
                new[..., :n] = last[..., :n]
            observation[self.state_key] = new
        return observation

    def launch_next_inference(self, observation: dict) -> _Pending:
        """Enqueues the next chunk's inference (asynchronous on a CUDA policy)."""
        observation = self._future_state(observation)
        self.launches.append({"chunk_index": self.chunk_index, "state": observation.get(self.state_key)})
        kw = {"incremental_input": self._incremental} if self.streaming else {}
        on_gpu = torch.cuda.is_available() and any(
            isinstance(v, torch.Tensor) and v.is_cuda for v in observation.values())
        if not on_gpu:
            chunk = self.policy.predict_action_chunk(observation, **kw)
            host = torch.as_tensor(chunk).detach().cpu()
            pending = _Pending(host[0] if host.dim() == 3 else host, None)
        else:
            if self.stream is None:
                self.stream = torch.cuda.Stream()
            self.stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(self.stream):
                chunk = self.policy.predict_action_chunk(observation, **kw)
                chunk = chunk[0] if chunk.dim() == 3 else chunk
                host = torch.empty(chunk.shape, dtype=chunk.dtype, pin_memory=True)
                host.copy_(chunk, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.stream)
            pending = _Pending(host, ev)
        if self.streaming:
            self._incremental = True
        return pending

    def wait(self) -> None:
        """Blocks until the pending inference (if any) has completed.  The
        policy's engine belongs to that inference until then: call this before
        using the policy outside the scheduler."""
        if self.next_chunk is not None and self.next_chunk.event is not None:
            self.next_chunk.event.synchronize()

    def get_action(self, observation: dict) -> np.ndarray:
        """The action to execute now (the control loop calls this once per step)."""
        if not self.is_running():  # bootstrap: the first chunk, synchronously
            self.current_chunk = self.launch_next_inference(observation).result()
        elif self.should_switch_chunk():
            self.current_chunk = self.next_chunk.result() if self.next_chunk is not None else None
            self.next_chunk = None
        if self.should_launch_next_inference():
            self.next_chunk = self.launch_next_inference(observation)
        action = self.get_current_action()
        self.chunk_index = (self.chunk_index + 1) % self.n_action_steps
        self.current_chunk = None if self.chunk_index == 0 else self.current_chunk
        return action


class PrefillDecodeStreams:
    """Prefill (source / frame update) and decode (action chunk) on separate
    CUDA streams, ordered through events (ConcurrentStreamingExecutor with
    use_cuda_streams=True)."""

    def __init__(self, device=None):
        self.prefill_stream = torch.cuda.Stream(device=device)
        self.decode_stream = torch.cuda.Stream(device=device)
        self.prefill_event = torch.cuda.Event()
        self.decode_event = torch.cuda.Event()
        self._prefilled = False

    def concurrent_prefill(self, prefill_func, wait: bool = False):
        """Runs prefill_func on the prefill stream (after the caller's pending
        work); with wait=True the caller's stream waits for it."""
        caller = torch.cuda.current_stream()
        with torch.cuda.stream(self.prefill_stream):
            self.prefill_stream.wait_stream(caller)
            result = prefill_func()
            self.prefill_event.record(self.prefill_stream)
        self._prefilled = True
        if wait:
            caller.wait_event(self.prefill_event)
        return result

    def concurrent_decode(self, decode_func, wait_for_prefill: bool = True):
        """Runs decode_func on the decode stream, after the last prefill when
        wait_for_prefill; the caller's stream then waits for the decode."""
        caller = torch.cuda.current_stream()
        with torch.cuda.stream(self.decode_stream):
            self.decode_stream.wait_stream(caller)
            if wait_for_prefill and self._prefilled:
                self.decode_stream.wait_event(self.prefill_event)
            result = decode_func()
            self.decode_event.record(self.decode_stream)
        caller.wait_event(self.decode_event)
        return result

    def synchronize_streams(self) -> None:
        self.prefill_event.synchronize()
        self.decode_event.synchronize()
