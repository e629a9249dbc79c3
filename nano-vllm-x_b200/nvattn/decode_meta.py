"""Decode-step metadata on the device (scope row f2).

Replaces ModelRunner.prepare_decode (nanovllm/engine/model_runner.py:172-188)
and, on the CUDA-graph path, the copies of its results into the graph's
static inputs (model_runner.py:204-210).

The reference turns five Python lists into five pinned tensors, copies each to
the GPU, then runs seven small copy/fill operations before the replay. Here the
host writes one record per sequence (last token, length, block table) into one
reused pinned buffer; ``nvattn_decode_prepare`` copies it to the device and one
kernel derives positions and slots and writes every output in place, including
the graph's padding rows (slot -1, context length 0).
"""
from __future__ import annotations

from array import array

import numpy as np
import torch

from . import _lib


_PADS: dict[int, array] = {}


def record_views(buf: np.ndarray, B: int, W: int):
    """The packed record's four arrays inside a uint8 buffer (layout of
    nvattn_decode_prepare): last_token int64[B], num_tokens int32[B],
    table_len int32[B], block_table int32[B*W]."""
    return (buf[:8 * B].view(np.int64), buf[8 * B:12 * B].view(np.int32),
            buf[12 * B:16 * B].view(np.int32), buf[16 * B:16 * B + 4 * B * W].view(np.int32))


def pack_record(buf: np.ndarray, last_tokens, num_tokens, tables,
                max_seqs: int, max_width: int) -> tuple[int, int]:
    """Write one record per sequence into ``buf`` (uint8); returns (B, W)."""
    B = len(tables)
    if not (len(last_tokens) == len(num_tokens) == B):
        raise ValueError("one last token, length and block table per sequence")
    if B == 0:
        raise ValueError("a decode step needs at least one sequence")
    if B > max_seqs:
        raise ValueError(f"{B} sequences > max_seqs {max_seqs}")
    tl = [len(t) for t in tables]
    W = max(tl)
    if W > max_width:
        raise ValueError(f"block table of {W} blocks > max_table_width {max_width}")
    tok, lens, tlen, flat = record_views(buf, B, W)
    tok[:] = last_tokens
    lens[:] = num_tokens
    tlen[:] = tl
    # rows padded with -1 to the widest table (model_runner.py:124-125)
    rows = array("i")
    for t, n in zip(tables, tl):
        if isinstance(t, list):
            rows.fromlist(t)
        else:
            rows.extend(t)
        pad = _PADS.get(W - n)
        if pad is None:
            pad = _PADS[W - n] = array("i", [-1] * (W - n))
        rows.extend(pad)
    flat[:] = np.frombuffer(rows, np.int32)
    return B, W


class DecodeMetadata:
    """Reusable packed buffers for up to ``max_seqs`` sequences whose block
    tables hold at most ``max_table_width`` blocks.

    ``pack(seqs)`` fills the pinned record from the engine's Sequence objects
    (``len(seq)``, ``seq.last_token``, ``seq.block_table``, as
    model_runner.py:177-181 reads them); ``launch(...)`` copies it and runs
    the kernel on the current stream. A record is not rewritten before the
    previous launch's copy has finished (an event guards it).
    """

    def __init__(self, max_seqs: int, max_table_width: int, block_size: int,
                 device: torch.device | str | int = "cuda"):
        if max_seqs <= 0 or max_table_width <= 0 or block_size <= 0:
            raise ValueError("max_seqs, max_table_width and block_size must be positive")
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("nvattn ops need CUDA tensors (no CPU fallback)")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.max_seqs, self.max_w, self.block_size = max_seqs, max_table_width, block_size
        nbytes = int(_lib.load().nvattn_decode_prepare_bytes(max_seqs, max_table_width))
        self.host = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
        self.dev = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        self._host_np = self.host.numpy()
        self._copied: torch.cuda.Event | None = None
        self.num_seqs = self.width = 0

    def pack_lists(self, last_tokens, num_tokens, tables) -> tuple[int, int]:
        """Pack plain lists: last token, len(seq) and block table per sequence."""
        if self._copied is not None:
            self._copied.synchronize()  # the previous record's copy has read the buffer
        B, W = pack_record(self._host_np, last_tokens, num_tokens, tables, self.max_seqs,
                           self.max_w)
        self.num_seqs, self.width = B, W
        return B, W

    def pack(self, seqs) -> tuple[int, int]:
        """Pack the engine's Sequence objects (model_runner.py:177-181);
        ``num_tokens`` is what ``len(seq)`` returns (sequence.py:33-34)."""
        return self.pack_lists([s.last_token for s in seqs], [s.num_tokens for s in seqs],
                               [s.block_table for s in seqs])

    def launch(self, pad_rows: int | None = None, *, input_ids=None, positions=None,
               slot_mapping=None, context_lens=None, block_tables=None, status=None) -> None:
        """Copy the packed record and write the outputs (any may be None).

        Rows [num_seqs, pad_rows) of slot_mapping / context_lens get -1 / 0;
        pad_rows defaults to num_seqs. block_tables is a (rows, cols) int32
        tensor with cols >= the packed width; only its first ``width``
        columns of the first ``num_seqs`` rows are written.
        """
        B, W = self.num_seqs, self.width
        if B == 0:
            raise ValueError("pack() a decode step first")
        pad_rows = B if pad_rows is None else int(pad_rows)
        checks = ((input_ids, torch.int64), (positions, torch.int64),
                  (slot_mapping, torch.int32), (context_lens, torch.int32))
        for t, dt in checks:
            if t is None:
                continue
            if t.device != self.device or t.dtype != dt or not t.is_contiguous() \
                    or t.numel() < pad_rows:
                raise ValueError(f"outputs must be contiguous {dt} CUDA tensors of >= {pad_rows} rows")
        for t in (input_ids, positions):
            if t is not None and t.numel() < B:
                raise ValueError("input_ids / positions need num_seqs rows")
        bt_stride = 0
        if block_tables is not None:
            if block_tables.device != self.device or block_tables.dtype != torch.int32 \
                    or block_tables.dim() != 2 or block_tables.stride(1) != 1 \
                    or block_tables.shape[0] < B or block_tables.shape[1] < W:
                raise ValueError("block_tables must be an int32 CUDA (rows, >= width) tensor")
            bt_stride = block_tables.stride(0)
        from .ops import _stream, status_tensor
        if status is None:
            status = status_tensor(self.device)

        def ptr(t):
            return t.data_ptr() if t is not None else None

        stream = _stream(self.device)
        _lib.call("nvattn_decode_prepare", self.host.data_ptr(), self.dev.data_ptr(), B, W,
                  self.block_size, pad_rows, ptr(input_ids), ptr(positions), ptr(slot_mapping),
                  ptr(context_lens), ptr(block_tables), bt_stride, ptr(status), stream)
        if self._copied is None:
            self._copied = torch.cuda.Event()
        self._copied.record(torch.cuda.current_stream(self.device))
