"""Sharded and streaming E-steps on top of the C ABI.

``ShardedEStep``: one process per GPU (torch.distributed, NCCL).  Each rank
owns a contiguous block of rows, runs the E-step on them, and the O(K D)
statistics of all ranks are summed by ONE all-reduce of a single packed buffer
``[Nk | mu_acc | sig]``.  logZ stays with the rank that owns the rows.  This is
the multi-GPU form of the reference's chunk-summing recipe (README.md:81-103),
which has no distributed code of its own.

``stream_estep``: the reference recipe for N larger than device memory
(README.md:81-103) -- host chunks are copied to the device through two pinned
staging buffers on a copy stream, overlapped with the E-step of the previous
chunk, and the statistics are accumulated in place (FGMM_FLAG_ACCUMULATE).

``resumable_stream_estep``: the same pass over rows [0, n_rows) read by a
callable, with its progress ``(next_row, Nk, mu_acc, sig, sum logZ)`` saved
to a checkpoint file every few chunks, so a pass that stops (a crash, a
pre-empted job) continues from the last checkpoint and ends with the
statistics an uninterrupted pass would have produced, bit for bit.

``generate_rows``: rows of the streaming configuration made on the device by
the library's counter-based generator, keyed by global row index, so every
sharding of the same global row range sees the same data.
"""

from __future__ import annotations

import dataclasses
import math
import os
from typing import Callable, Iterable, Optional

import torch
import torch.distributed as dist

import _fgmm_lib as L

VARIANTS = {"iso": L.FGMM_VARIANT_ISO, "diag": L.FGMM_VARIANT_DIAG, "full": L.FGMM_VARIANT_FULL}


def sig_shape(variant: str, K: int, D: int):
    return (K,) if variant == "iso" else (K, D) if variant == "diag" else (K, D, D)


def packed_stats(variant: str, K: int, D: int, device, dtype=torch.float32):
    """One contiguous buffer and its (Nk, mu_acc, sig) views."""
    n_sig = math.prod(sig_shape(variant, K, D))
    buf = torch.empty(K + K * D + n_sig, device=device, dtype=dtype)
    Nk = buf[:K]
    mu_acc = buf[K:K + K * D].view(K, D)
    sig = buf[K + K * D:].view(sig_shape(variant, K, D))
    return buf, (Nk, mu_acc, sig)


def shard_rows(N: int, rank: int, world: int):
    """Contiguous row range [lo, hi) of ``rank`` (sizes differ by at most 1)."""
    base, extra = divmod(N, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def _local_estep(variant: str):
    def run(X, mu, cov, log_pi, out):
        return L.estep(VARIANTS[variant], X, mu, cov, log_pi, out=out)
    return run


class ShardedEStep:
    """E-step over row shards held by the ranks of a process group.

    ``estep_fn(X, mu, cov, log_pi, out)`` computes one rank's local E-step into
    ``out = (logZ, Nk, mu_acc, sig)``; it defaults to the CUDA library.  (Tests
    on CPU ranks pass a CPU function; the product path has no CPU fallback.)
    """

    def __init__(self, variant: str = "iso", group=None,
                 estep_fn: Optional[Callable] = None):
        if variant not in VARIANTS:
            raise ValueError(f"unknown variant {variant!r}")
        self.variant = variant
        self.group = group
        self.estep_fn = estep_fn or _local_estep(variant)
        self._buf = None

    def __call__(self, X_local: torch.Tensor, mu: torch.Tensor, cov: torch.Tensor,
                 log_pi: torch.Tensor):
        K, D = mu.shape
        dev = X_local.device
        if self._buf is None or self._buf[0].device != dev or \
                self._buf[0].numel() != K + K * D + math.prod(sig_shape(self.variant, K, D)):
            self._buf = packed_stats(self.variant, K, D, dev)
        buf, (Nk, mu_acc, sig) = self._buf
        logZ = torch.empty(X_local.shape[0], device=dev, dtype=torch.float32)
        self.estep_fn(X_local, mu, cov, log_pi, (logZ, Nk, mu_acc, sig))
        if dist.is_available() and dist.is_initialized():
            dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=self.group)
        return logZ, Nk, mu_acc, sig


def stream_estep(chunks: Iterable[torch.Tensor], mu: torch.Tensor, cov: torch.Tensor,
                 log_pi: torch.Tensor, variant: str = "iso", device=None,
                 keep_logZ: bool = False, init=None):
    """E-step over host chunks (each (n_i, D) float32, ideally pinned).

    Copies chunk i+1 on a side stream while chunk i is processed; statistics
    are accumulated on the device, starting from ``init = (Nk, mu_acc, sig)``
    when given (a resumed pass) and from zero otherwise.  Returns
    (logZ or None, Nk, mu_acc, sig).
    """
    device = torch.device(device or "cuda")
    K, D = mu.shape
    mu = mu.to(device)
    cov = cov.to(device)
    log_pi = log_pi.to(device)
    _, (Nk, mu_acc, sig) = packed_stats(variant, K, D, device)
    if init is not None:
        for dst, src in zip((Nk, mu_acc, sig), init):
            dst.copy_(src.reshape(dst.shape))
    copy_stream = torch.cuda.Stream(device)
    compute = torch.cuda.current_stream(device)
    logZ_parts = []
    # two device staging buffers, reused for every chunk (grown if a larger
    # chunk comes): no allocation per chunk, and no cross-stream frees
    bufs = [None, None]
    staged = [None, None]
    events = [torch.cuda.Event(), torch.cuda.Event()]
    first = True
    it = iter(chunks)
    nxt = next(it, None)
    slot = 0

    def stage(chunk, s):
        n = chunk.shape[0]
        b = bufs[s]
        if b is None or b.shape[0] < n or b.dtype != chunk.dtype or b.shape[1:] != chunk.shape[1:]:
            # allocated on the compute stream, whose E-step is the last user
            bufs[s] = b = torch.empty((n,) + tuple(chunk.shape[1:]), device=device,
                                      dtype=chunk.dtype)
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_stream(compute)  # buffer s free once its last E-step ran
            staged[s] = b[:n]
            staged[s].copy_(chunk, non_blocking=True)
            events[s].record(copy_stream)

    if nxt is not None:
        stage(nxt, slot)
    while nxt is not None:
        cur_slot = slot
        nxt = next(it, None)
        slot ^= 1
        if nxt is not None:
            stage(nxt, slot)
        compute.wait_event(events[cur_slot])
        Xd = staged[cur_slot]
        logZ = torch.empty(Xd.shape[0], device=device, dtype=torch.float32)
        L.estep(VARIANTS[variant], Xd, mu, cov, log_pi, out=(logZ, Nk, mu_acc, sig),
                accumulate=init is not None or not first)
        first = False
        if keep_logZ:
            logZ_parts.append(logZ)
    if first and init is None:  # no chunk at all
        Nk.zero_()
        mu_acc.zero_()
        sig.zero_()
    logZ = torch.cat(logZ_parts) if keep_logZ and logZ_parts else None
    return logZ, Nk, mu_acc, sig


@dataclasses.dataclass
class StreamState:
    """Progress of a resumable streamed E-step: rows [0, next_row) are in the
    statistics (host fp32 tensors) and in sum_logZ (float64 on the host)."""
    variant: str
    n_rows: int
    chunk_rows: int
    next_row: int
    Nk: torch.Tensor
    mu_acc: torch.Tensor
    sig: torch.Tensor
    sum_logZ: float = 0.0

    @classmethod
    def start(cls, variant: str, n_rows: int, chunk_rows: int, K: int, D: int) -> "StreamState":
        shape = sig_shape(variant, K, D)
        return cls(variant, n_rows, chunk_rows, 0, torch.zeros(K), torch.zeros(K, D),
                   torch.zeros(shape))

    @property
    def done(self) -> bool:
        return self.next_row >= self.n_rows

    def save(self, path: str) -> None:
        """Atomic: written to a temporary file, then renamed over ``path``."""
        tmp = f"{path}.tmp"
        torch.save({"variant": self.variant, "n_rows": self.n_rows,
                    "chunk_rows": self.chunk_rows, "next_row": self.next_row,
                    "Nk": self.Nk, "mu_acc": self.mu_acc, "sig": self.sig,
                    "sum_logZ": self.sum_logZ}, tmp)
        os.replace(tmp, path)

    @classmethod
    def load(cls, path: str) -> "StreamState":
        d = torch.load(path, map_location="cpu", weights_only=True)
        return cls(d["variant"], int(d["n_rows"]), int(d["chunk_rows"]), int(d["next_row"]),
                   d["Nk"], d["mu_acc"], d["sig"], float(d["sum_logZ"]))


def resumable_stream_estep(read_rows: Callable[[int, int], torch.Tensor], n_rows: int,
                           mu: torch.Tensor, cov: torch.Tensor, log_pi: torch.Tensor,
                           variant: str = "iso", chunk_rows: int = 1 << 20,
                           checkpoint_path: Optional[str] = None, checkpoint_every: int = 8,
                           state: Optional[StreamState] = None,
                           logz_sink: Optional[Callable[[int, torch.Tensor], None]] = None,
                           device=None, window_fn: Optional[Callable] = None) -> StreamState:
    """Streamed E-step over rows [0, n_rows) with checkpoints (N larger than
    device memory, README.md:81-103, plus resume).

    read_rows(row0, n) returns host rows [row0, row0+n) as an (n, D) float32
    tensor (pinned for overlap).  Rows go through ``stream_estep`` in windows
    of ``checkpoint_every`` chunks of ``chunk_rows``; after each window the
    statistics come back to the host and, with ``checkpoint_path``, the state
    is saved.  ``state`` (or an existing checkpoint file) resumes a pass: the
    chunking must be the one the state was made with.  logz_sink(row0, logZ)
    receives each window's logZ.  ``window_fn(chunks, mu, cov, log_pi, init)``
    replaces the device E-step (CPU tests only; default ``stream_estep``).
    Returns the final state."""
    K, D = mu.shape
    if state is None and checkpoint_path is not None and os.path.exists(checkpoint_path):
        state = StreamState.load(checkpoint_path)
    if state is None:
        state = StreamState.start(variant, n_rows, chunk_rows, K, D)
    if (state.variant, state.n_rows, state.chunk_rows) != (variant, n_rows, chunk_rows):
        raise ValueError("resume state was made for another pass: "
                         f"{(state.variant, state.n_rows, state.chunk_rows)} != "
                         f"{(variant, n_rows, chunk_rows)}")
    if state.next_row % chunk_rows != 0 and state.next_row < n_rows:
        raise ValueError("resume state is not on a chunk boundary")
    if window_fn is None:
        def window_fn(chunks, mu_, cov_, lpi_, init):
            return stream_estep(chunks, mu_, cov_, lpi_, variant=variant, device=device,
                                keep_logZ=True, init=init)
    while not state.done:
        row0 = state.next_row
        starts = range(row0, min(n_rows, row0 + checkpoint_every * chunk_rows), chunk_rows)
        chunks = [read_rows(r, min(chunk_rows, n_rows - r)) for r in starts]
        logZ, Nk, mu_acc, sig = window_fn(chunks, mu, cov, log_pi,
                                          (state.Nk, state.mu_acc, state.sig))
        logZ_h = logZ.double().cpu()
        state.Nk, state.mu_acc, state.sig = Nk.cpu(), mu_acc.cpu(), sig.cpu()
        state.sum_logZ += float(logZ_h.sum())
        state.next_row = min(n_rows, starts[-1] + chunk_rows)
        if logz_sink is not None:
            logz_sink(row0, logZ.cpu())
        if checkpoint_path is not None:
            state.save(checkpoint_path)
    return state


def mixture_centres(K: int, D: int, seed: int, device) -> torch.Tensor:
    """Centres ~ N(0, 4 I) of the streaming mixture (the C2 recipe)."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    return (2.0 * torch.randn(K, D, generator=g)).to(device)


def generate_rows(row0: int, nrows: int, centres: torch.Tensor, seed: int,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Rows [row0, row0+nrows) of the streaming mixture, on centres' device."""
    K, D = centres.shape
    if out is None:
        out = torch.empty(nrows, D, device=centres.device, dtype=torch.float32)
    return L.generate_iso_rows(out, centres, seed, row0=row0)


def generate_row_ids(row_ids: torch.Tensor, centres: torch.Tensor, seed: int) -> torch.Tensor:
    """The given global rows of the streaming mixture (e.g. to pick means)."""
    K, D = centres.shape
    out = torch.empty(row_ids.numel(), D, device=centres.device, dtype=torch.float32)
    return L.generate_iso_rows(out, centres, seed, row_ids=row_ids)


def pick_mean_rows(N: int, K: int, seed: int) -> torch.Tensor:
    """K distinct global row ids in [0, N) (``mu`` = K random rows of X)."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed + 1)
    if N <= 50_000_000:
        return torch.randperm(N, generator=g)[:K]
    picked = torch.unique(torch.randint(0, N, (4 * K,), generator=g))
    return picked[torch.randperm(picked.numel(), generator=g)[:K]]
