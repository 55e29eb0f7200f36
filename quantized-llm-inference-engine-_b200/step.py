"""Decode-step metadata kept on the device (``llmopt_decode_step_advance``).

Replaces the per-step host build of ``ModelRunner._build_decode`` +
``_finalize`` (src/llmopt/engine/model_runner.py:169-230), which loops over
the requests in Python, allocates a fresh ``-1`` table and copies every row to
the device separately.  Here the block table, context lengths, write offsets
and positions of the running sequences live on the device; the host records
only what changed since the last step (a sequence admitted, a block appended,
a sequence released) and one launch applies the changes and advances every
row by one token.  Rows stay compact: releasing a sequence moves the last row
into its place.  Since the update count is read on the device, a CUDA graph
that captured a decode step (this advance, the rotary append and attention)
replays with any number of updates up to ``capacity``.
"""

from __future__ import annotations

import torch

from . import _lib
from . import _runtime as rt


class StepLedger:
    """Host bookkeeping of the device step state (no device memory): which
    sequence holds which row, how many blocks each row has, and the update
    records (op, row, a, b) the next step must apply, in order."""

    def __init__(self, max_seqs: int, max_blocks: int) -> None:
        self.max_seqs = max_seqs
        self.max_blocks = max_blocks
        self.pending: list[tuple[int, int, int, int]] = []
        self.order: list = []                  # row -> sequence id
        self.rows: dict = {}                   # sequence id -> row
        self.nblocks: dict = {}                # sequence id -> blocks in its row

    def admit(self, seq_id, blocks, committed: int) -> int:
        if seq_id in self.rows:
            raise ValueError(f"sequence {seq_id!r} is already running")
        if len(self.order) >= self.max_seqs:
            raise ValueError("no free row")
        blocks = [int(b) for b in blocks]
        if len(blocks) > self.max_blocks:
            raise ValueError(f"{len(blocks)} blocks exceed the table width {self.max_blocks}")
        row = len(self.order)
        self.order.append(seq_id)
        self.rows[seq_id] = row
        self.nblocks[seq_id] = len(blocks)
        self.pending.append((_lib.STEP_ADMIT, row, int(committed), 0))
        for c, b in enumerate(blocks):
            self.pending.append((_lib.STEP_SET_BLOCK, row, c, b))
        return row

    def append_block(self, seq_id, block_id: int) -> None:
        row = self.rows[seq_id]
        col = self.nblocks[seq_id]
        if col >= self.max_blocks:
            raise ValueError(f"sequence {seq_id!r} exceeds the table width {self.max_blocks}")
        self.nblocks[seq_id] = col + 1
        self.pending.append((_lib.STEP_SET_BLOCK, row, col, int(block_id)))

    def release(self, seq_id) -> None:
        row = self.rows.pop(seq_id)
        self.nblocks.pop(seq_id)
        last = len(self.order) - 1
        if row != last:
            moved = self.order[last]
            self.pending.append((_lib.STEP_MOVE, row, last, 0))
            self.order[row] = moved
            self.rows[moved] = row
        self.order.pop()

    def take(self) -> list:
        """The records of the next step (and forget them)."""
        out, self.pending = self.pending, []
        return out


class DecodeStepState:
    """Device-resident ``block_ids`` / ``context_lens`` / ``token_offsets`` /
    ``positions`` for up to ``max_seqs`` decoding sequences.

    Per step the values of row r match the reference's for the same request:
    position = token offset = committed tokens, context length = committed + 1,
    table row = the request's blocks, ``-1`` padded (model_runner.py:169-230).
    """

    def __init__(self, max_seqs: int, max_blocks: int, device=None, capacity: int = 4096) -> None:
        if max_seqs < 1 or max_blocks < 1 or capacity < 1:
            raise ValueError("max_seqs, max_blocks and capacity must be >= 1")
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        rt.require_cuda(torch.empty(0, device=self.device), "DecodeStepState")
        self.max_seqs = max_seqs
        self.max_blocks = max_blocks
        self.capacity = capacity
        self.block_ids = torch.full((max_seqs, max_blocks), -1, dtype=torch.int32,
                                    device=self.device)
        self.context_lens = torch.zeros(max_seqs, dtype=torch.int64, device=self.device)
        self.token_offsets = torch.zeros(max_seqs, dtype=torch.int64, device=self.device)
        self.positions = torch.zeros(max_seqs, dtype=torch.int64, device=self.device)
        # Two pinned staging buffers: the one being filled was last copied two
        # steps ago, and its event says whether that copy has left it yet.
        self._hosts = [torch.zeros(1 + 4 * capacity, dtype=torch.int64, pin_memory=True)
                       for _ in range(2)]
        self._copied = [None, None]
        self._turn = 0
        self._dev = torch.zeros(1 + 4 * capacity, dtype=torch.int64, device=self.device)
        self.ledger = StepLedger(max_seqs, max_blocks)

    # -- scheduling decisions (host) ---------------------------------------------
    @property
    def order(self) -> list:
        """Sequence id of every running row."""
        return self.ledger.order

    @property
    def _pending(self) -> list:
        return self.ledger.pending

    @property
    def _nblocks(self) -> dict:
        return self.ledger.nblocks

    def admit(self, seq_id, blocks, committed: int) -> int:
        """A sequence joins with ``committed`` tokens already in its ``blocks``."""
        return self.ledger.admit(seq_id, blocks, committed)

    def append_block(self, seq_id, block_id: int) -> None:
        """The sequence's next token needs one more block."""
        self.ledger.append_block(seq_id, block_id)

    def release(self, seq_id) -> None:
        """The sequence finished; the last row moves into its place."""
        self.ledger.release(seq_id)

    def row_of(self, seq_id) -> int:
        return self.ledger.rows[seq_id]

    # -- the step (device) ---------------------------------------------------------
    def step(self):
        """Apply the recorded changes and advance every running row by one token.

        Returns the ``(block_ids, context_lens, token_offsets, positions)`` views
        of the active rows, ready for ``rope_kv_append`` and ``PagedAttention``.
        """
        self.stage()
        self.launch()
        b = len(self.order)
        return (self.block_ids[:b], self.context_lens[:b], self.token_offsets[:b],
                self.positions[:b])

    def stage(self) -> None:
        """Copy the recorded changes into the device update buffer (stream
        ordered, no host sync unless the staging buffer in turn is still being
        copied from two steps ago); ``launch`` or a graph replay applies them."""
        records = self.ledger.take()
        n = len(records)
        if n > self.capacity:
            raise ValueError(f"{n} updates exceed the capacity {self.capacity}")
        k = self._turn
        self._turn ^= 1
        if self._copied[k] is not None:
            self._copied[k].synchronize()
        host = self._hosts[k]
        host[0] = n
        if n:
            host[1:1 + 4 * n] = torch.tensor(records, dtype=torch.int64).reshape(-1)
        self._dev[:1 + 4 * n].copy_(host[:1 + 4 * n], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self._copied[k] = ev

    def launch(self, batch: int | None = None) -> None:
        """The advance kernel alone, on the updates already in device memory
        (what a captured graph replays)."""
        err = rt.err_word(self.device)
        st = _lib.lib().llmopt_decode_step_advance(
            self._dev.data_ptr(), self.capacity, self.block_ids.data_ptr(), self.max_blocks,
            self.block_ids.stride(0), self.context_lens.data_ptr(), self.token_offsets.data_ptr(),
            self.positions.data_ptr(), self.max_seqs, len(self.order) if batch is None else batch,
            err.data_ptr(), rt.stream_handle(self.device))
        _lib.check(st, "DecodeStepState.step")
