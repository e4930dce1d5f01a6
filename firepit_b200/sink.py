"""Submission policies (crates/firepit-kernels/src/sink.rs).

A sink decides how a launch is issued: ``Eager`` runs it and synchronises
(sink.rs:82-92), ``Graph`` records it into a CUDA graph captured on a side
stream (sink.rs:94-105), ``Traced`` brackets each op with CUDA events and
keeps per-kind totals (sink.rs:24-80, 107-124), ``Dry`` records the op kinds
without launching anything (sink.rs:126-135).
"""
from __future__ import annotations

from collections import defaultdict
from dataclasses import dataclass, field
from typing import Callable


def _stream_handle(stream) -> int:
    import torch
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)


class Sink:
    def run(self, kind: str, launch: Callable[[int], None]) -> None:  # pragma: no cover - interface
        raise NotImplementedError


class Eager(Sink):
    """Launch on ``stream`` (torch stream or raw handle) and wait for it."""

    def __init__(self, stream=None):
        self.stream = stream

    def run(self, kind: str, launch: Callable[[int], None]) -> None:
        import torch
        launch(_stream_handle(self.stream))
        if self.stream is None:
            torch.cuda.current_stream().synchronize()
        elif hasattr(self.stream, "synchronize"):
            self.stream.synchronize()
        else:
            torch.cuda.synchronize()


class Async(Sink):
    """Launch on ``stream`` without synchronising (the graph-capturable form)."""

    def __init__(self, stream=None):
        self.stream = stream

    def run(self, kind: str, launch: Callable[[int], None]) -> None:
        launch(_stream_handle(self.stream))


@dataclass
class Span:
    kind: str
    gpu_ms: float


@dataclass
class Traced(Sink):
    """Times every op with CUDA events on the launching stream."""

    stream: object = None
    spans: list = field(default_factory=list)

    def run(self, kind: str, launch: Callable[[int], None]) -> None:
        import torch
        s = self.stream or torch.cuda.current_stream()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(s)
        launch(_stream_handle(s))
        end.record(s)
        end.synchronize()
        self.spans.append(Span(kind, start.elapsed_time(end)))

    def summary(self) -> dict[str, tuple[int, float]]:
        out: dict[str, list] = defaultdict(lambda: [0, 0.0])
        for sp in self.spans:
            out[sp.kind][0] += 1
            out[sp.kind][1] += sp.gpu_ms
        return {k: (v[0], v[1]) for k, v in out.items()}


@dataclass
class Dry(Sink):
    """Records op kinds; launches nothing (sink.rs:126-135)."""

    kinds: list = field(default_factory=list)

    def run(self, kind: str, launch: Callable[[int], None]) -> None:
        self.kinds.append(kind)


class Graph(Sink):
    """Captures every op into one CUDA graph; ``replay()`` launches it."""

    def __init__(self):
        import torch
        self.graph = torch.cuda.CUDAGraph()
        self.stream = torch.cuda.Stream()
        self._ctx = None

    def __enter__(self):
        import torch
        self._ctx = torch.cuda.graph(self.graph, stream=self.stream)
        self._ctx.__enter__()
        return self

    def __exit__(self, *exc):
        return self._ctx.__exit__(*exc)

    def run(self, kind: str, launch: Callable[[int], None]) -> None:
        import torch
        launch(torch.cuda.current_stream().cuda_stream)

    def replay(self) -> None:
        self.graph.replay()
