"""Training data into steps: chat JSONL to scored token sequences, the token-budget batcher and the step's
input rows.

``ChatData`` mirrors the reference's ``r97::ChatData`` (include/r97/chatdata.h, src/chatdata.cpp): one
conversation a JSONL line, kept through its last assistant turn, trailing assistant turns dropped until the
render fits, and each assistant turn's generated tokens scored (libr97host.so, host/chatdata.cpp). The
reference renders with its container's chat template and tokenizer (radiance, not in this tree); the
library's renderer is ChatML over a byte vocabulary, the form the reference's own mask test states its
expectations in.

``Batcher`` mirrors the reference's ``r97::Batcher`` (include/r97/batcher.h:46-100, src/batcher.cpp): one
``TokenSeq`` per example, ``BatcherConfig(token_budget, devices, seed)``, ``next()`` handing out one
sub-batch per device, ``steps_in_epoch``, ``position`` / ``seek`` / ``reset`` and ``skipped``. The plan is
computed by libr97host.so (``r97host_batcher_*``, r97training_b200/host/batcher.cpp), which hands out the
same sub-batches of the same sequences in the same order as the reference for every (seed, epoch), so a
saved position resumes identically on either.

``step_rows`` lays one sub-batch into the fixed ``[rows, seq]`` frame ``TrainStep.run`` takes: a sequence a
row, padded, with next-token targets where the sequence scores the token (``TokenSeq.score``, include/r97/
batch.h: ``score[i] == 1`` when token i is a target predicted at position i - 1) and -1 elsewhere."""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field

import numpy as np

from . import build as _build

_host = None


def host():
    """libr97host.so, bound for the batcher entry points."""
    global _host
    if _host is None:
        if not os.path.exists(_build.HOSTLIB):
            _build.build_all()
        lib = ctypes.CDLL(_build.HOSTLIB)
        vp, i64, p64 = ctypes.c_void_p, ctypes.c_int64, ctypes.POINTER(ctypes.c_int64)
        lib.r97host_batcher_create.restype = vp
        lib.r97host_batcher_create.argtypes = [vp, i64, i64, ctypes.c_int32, ctypes.c_uint64]
        lib.r97host_batcher_destroy.argtypes = [vp]
        lib.r97host_batcher_next.restype = ctypes.c_int32
        lib.r97host_batcher_next.argtypes = [vp, vp, vp, i64]
        lib.r97host_batcher_steps_in_epoch.restype = i64
        lib.r97host_batcher_steps_in_epoch.argtypes = [vp, i64]
        lib.r97host_batcher_position.argtypes = [vp, p64, p64]
        lib.r97host_batcher_seek.argtypes = [vp, i64, i64]
        lib.r97host_batcher_reset.argtypes = [vp]
        lib.r97host_batcher_skipped.restype = i64
        lib.r97host_batcher_skipped.argtypes = [vp, vp, i64]
        lib.r97host_batcher_skipped_tokens.restype = i64
        lib.r97host_batcher_skipped_tokens.argtypes = [vp]
        lib.r97host_batcher_error.restype = ctypes.c_char_p
        lib.r97host_chatdata_create_chatml_bytes.restype = vp
        lib.r97host_chatdata_destroy.argtypes = [vp]
        lib.r97host_chatdata_read.restype = ctypes.c_int32
        lib.r97host_chatdata_read.argtypes = [vp, ctypes.c_char_p, i64, ctypes.c_int32, p64]
        lib.r97host_chatdata_read_file.restype = ctypes.c_int32
        lib.r97host_chatdata_read_file.argtypes = [vp, ctypes.c_char_p, ctypes.c_int32, p64]
        lib.r97host_chatdata_line.restype = ctypes.c_int32
        lib.r97host_chatdata_line.argtypes = [vp, ctypes.c_char_p, i64, ctypes.c_int32, vp, vp, i64, p64]
        lib.r97host_chatdata_count.restype = i64
        lib.r97host_chatdata_count.argtypes = [vp]
        lib.r97host_chatdata_seq_len.restype = i64
        lib.r97host_chatdata_seq_len.argtypes = [vp, i64]
        lib.r97host_chatdata_seq.argtypes = [vp, i64, vp, vp]
        lib.r97host_chatdata_error.restype = ctypes.c_char_p
        lib.r97host_chatdata_error.argtypes = [vp]
        _host = lib
    return _host


@dataclass
class TokenSeq:
    """One example: token ids and, per token, 1 where it is a target predicted at the position before."""
    ids: list = field(default_factory=list)
    score: list = field(default_factory=list)


# ChatData outcomes (include/r97/chatdata.h ChatDataOutcome)
KEPT, SHORTENED, SKIPPED, ERROR = 0, 1, 2, 3
IM_START, IM_END = 256, 257  # the ChatML byte renderer's two control tokens


class ChatDataError(RuntimeError):
    pass


class ChatData:
    """Chat JSONL to TokenSeqs with the assistant loss mask (the reference's r97::ChatData), over the ChatML
    byte-vocabulary renderer. ``read`` / ``read_file`` return the kept sequences and add the outcome counts
    into ``stats`` (conversations, kept, shortened, skipped, tokens, scored); a malformed line raises
    ChatDataError("line N: ...") after the lines before it were kept."""

    DEFAULT_MAX_TOKENS = 4096
    STATS = ("conversations", "kept", "shortened", "skipped", "tokens", "scored")

    def __init__(self):
        self._lib = host()
        self._h = self._lib.r97host_chatdata_create_chatml_bytes()
        self._taken = 0
        self.stats = dict.fromkeys(self.STATS, 0)

    def __del__(self):
        if getattr(self, "_h", None):
            self._lib.r97host_chatdata_destroy(self._h)
            self._h = None

    def _error(self):
        return self._lib.r97host_chatdata_error(self._h).decode()

    def _new(self):
        out = []
        n = int(self._lib.r97host_chatdata_count(self._h))
        for i in range(self._taken, n):
            k = int(self._lib.r97host_chatdata_seq_len(self._h, i))
            ids = np.zeros(k, np.int32)
            score = np.zeros(k, np.uint8)
            self._lib.r97host_chatdata_seq(self._h, i, ids.ctypes.data, score.ctypes.data)
            out.append(TokenSeq(ids.tolist(), score.tolist()))
        self._taken = n
        return out

    def _count(self, st):
        for k, v in zip(self.STATS, st):
            self.stats[k] += int(v)

    def read(self, text: str, max_tokens: int = DEFAULT_MAX_TOKENS):
        b = text.encode()
        st = (ctypes.c_int64 * 6)()
        ok = self._lib.r97host_chatdata_read(self._h, b, len(b), max_tokens, st)
        self._count(st)
        seqs = self._new()
        if not ok:
            raise ChatDataError(self._error())
        return seqs

    def read_file(self, path: str, max_tokens: int = DEFAULT_MAX_TOKENS):
        st = (ctypes.c_int64 * 6)()
        ok = self._lib.r97host_chatdata_read_file(self._h, os.fsencode(path), max_tokens, st)
        self._count(st)
        seqs = self._new()
        if not ok:
            raise ChatDataError(self._error())
        return seqs

    def line(self, text: str, max_tokens: int = DEFAULT_MAX_TOKENS):
        """One conversation: (outcome, TokenSeq); the sequence is not appended to the read ones."""
        b = text.encode()
        n = ctypes.c_int64()
        cap = max(16, 4 * len(b) + 64)
        ids = np.zeros(cap, np.int32)
        score = np.zeros(cap, np.uint8)
        o = int(self._lib.r97host_chatdata_line(self._h, b, len(b), max_tokens, ids.ctypes.data, score.ctypes.data,
                                                cap, ctypes.byref(n)))
        if o == ERROR:
            raise ChatDataError(self._error())
        k = min(int(n.value), cap)
        return o, TokenSeq(ids[:k].tolist(), score[:k].tolist())

    def render(self, messages, max_tokens: int = DEFAULT_MAX_TOKENS):
        """A conversation given as [(role, content), ...] or [{"role", "content"}, ...]."""
        import json
        msgs = [m if isinstance(m, dict) else {"role": m[0], "content": m[1]} for m in messages]
        return self.line(json.dumps({"messages": msgs}), max_tokens)


@dataclass
class BatcherConfig:
    token_budget: int = 0  # tokens per sub-batch, not per step
    devices: int = 1       # sub-batches per step
    seed: int = 0          # the shuffle's seed; same seed, same batches


@dataclass
class Position:
    epoch: int = 0
    step: int = 0


class Batcher:
    """Token-budget batches over tokenised sequences (the reference's r97::Batcher). Raises ValueError
    where the reference throws std::invalid_argument (a budget <= 0, fewer than one device)."""

    def __init__(self, sequences, config: BatcherConfig):
        self._seqs = list(sequences)
        self._cfg = config
        lens = np.ascontiguousarray([len(s.ids) for s in self._seqs], dtype=np.int64)
        self._lens = lens
        lib = host()
        h = lib.r97host_batcher_create(lens.ctypes.data if len(lens) else None, len(lens), int(config.token_budget),
                                       int(config.devices), int(config.seed) & (2**64 - 1))
        if not h:
            raise ValueError(lib.r97host_batcher_error().decode())
        self._h = h
        self._counts = np.zeros(max(int(config.devices), 1), dtype=np.int64)
        self._idx = np.zeros(max(len(lens), 1), dtype=np.int64)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            host().r97host_batcher_destroy(h)
            self._h = None

    def next_indices(self):
        """The step at the position as input indices, one list a sub-batch; None at the epoch's end."""
        n = host().r97host_batcher_next(self._h, self._counts.ctypes.data, self._idx.ctypes.data, len(self._idx))
        if n < 0:
            raise RuntimeError(host().r97host_batcher_error().decode())
        if n == 0:
            return None
        out, o = [], 0
        for d in range(n):
            c = int(self._counts[d])
            out.append([int(i) for i in self._idx[o:o + c]])
            o += c
        return out

    def next(self):
        """The next step: one list of TokenSeq a device (Batcher::next); None at the epoch's end, consuming
        nothing -- ``seek(Position(epoch + 1, 0))`` moves on, ``reset()`` back to the first."""
        step = self.next_indices()
        return None if step is None else [[self._seqs[i] for i in sub] for sub in step]

    def steps_in_epoch(self, epoch: int) -> int:
        return int(host().r97host_batcher_steps_in_epoch(self._h, int(epoch)))

    def position(self) -> Position:
        e, s = ctypes.c_int64(), ctypes.c_int64()
        host().r97host_batcher_position(self._h, ctypes.byref(e), ctypes.byref(s))
        return Position(e.value, s.value)

    def seek(self, p: Position) -> None:
        host().r97host_batcher_seek(self._h, int(p.epoch), int(p.step))

    def reset(self) -> None:
        host().r97host_batcher_reset(self._h)

    def skipped(self) -> list:
        n = host().r97host_batcher_skipped(self._h, None, 0)
        out = np.zeros(max(n, 1), dtype=np.int64)
        host().r97host_batcher_skipped(self._h, out.ctypes.data, n)
        return [int(i) for i in out[:n]]

    def skipped_tokens(self) -> int:
        return int(host().r97host_batcher_skipped_tokens(self._h))

    def sequences(self):
        return self._seqs

    def config(self) -> BatcherConfig:
        return self._cfg


def step_rows(batch, rows: int, seq: int, pad_id: int = 0):
    """One sub-batch laid into the step's [rows, seq] frame: (ids int32 [rows, seq], targets int32
    [rows * seq], scored). Row r holds sequence r, padded with pad_id; position p of a row targets token
    p + 1 when the sequence scores it, else -1 (padding, unscored tokens, each row's last position).
    ValueError when the sub-batch has more sequences than rows or a sequence is longer than seq."""
    if len(batch) > rows:
        raise ValueError(f"step_rows: {len(batch)} sequences for {rows} rows")
    ids = np.full((rows, seq), pad_id, dtype=np.int32)
    tgt = np.full((rows, seq), -1, dtype=np.int32)
    for r, s in enumerate(batch):
        n = len(s.ids)
        if n > seq:
            raise ValueError(f"step_rows: a sequence of {n} tokens for rows of {seq}")
        if len(s.score) != n:
            raise ValueError("step_rows: score and ids differ in length")
        ids[r, :n] = np.asarray(s.ids, dtype=np.int32)
        if n > 1:
            sc = np.asarray(s.score[1:], dtype=np.uint8) != 0
            tgt[r, :n - 1] = np.where(sc, ids[r, 1:n], -1)
    return ids, tgt.reshape(-1), int((tgt >= 0).sum())
