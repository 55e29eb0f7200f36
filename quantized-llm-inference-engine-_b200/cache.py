"""``PagedKVCache`` backed by the B200 kernels (drop-in for ``llmopt.cache``).

Same constructor, attributes and methods as the reference's
``src/llmopt/cache/paged_cache.py:131-331``; storage is the same
``[num_layers, num_blocks, block_size, num_kv_heads, head_dim]`` pair of
tensors (``key_cache`` / ``value_cache``), allocated once in HBM and never
moved.  ``write`` / ``write_decode`` / ``gather`` run as single CUDA kernels
with no host synchronisation (``gather`` syncs once to size its output, as
the reference does at paged_cache.py:282).

Differences from the reference, all deliberate:

* storage must be on a CUDA device (``device=None`` means the current one;
  a CPU device raises): there is no CPU path;
* a block id >= ``num_blocks`` reached by ``write`` / ``gather`` is skipped and
  flagged on the device instead of raising (``LLMOPT_B200_CHECK=1`` restores
  the ``IndexError`` at the cost of a sync).

FP8 storage (``dtype=torch.float8_e4m3fn``), beyond the reference (which only
names the dtype, src/llmopt/utils/misc.py:33-34): ``key_cache`` /
``value_cache`` hold e4m3 codes in the same layout, and ``key_scale`` /
``value_scale`` hold one fp32 scale per (token, head) row,
``[num_layers, num_blocks, num_kv_heads, block_size]``; a value is code *
scale.  ``write`` / ``write_decode`` quantize each appended row with its own
scale (amax / 448), and ``gather`` returns the dequantized values in fp32.
"""

from __future__ import annotations

import torch

from . import _lib
from . import _runtime as rt


class PagedKVCache:
    """Fixed-capacity paged key/value cache shared by all layers (HBM-resident)."""

    def __init__(
        self,
        num_layers: int,
        num_blocks: int,
        block_size: int,
        num_kv_heads: int,
        head_dim: int,
        dtype: torch.dtype = torch.float16,
        device: torch.device | str | None = None,
    ) -> None:
        if num_layers < 1:
            raise ValueError("num_layers must be >= 1")
        if num_blocks < 1 or block_size < 1:
            raise ValueError("num_blocks and block_size must be >= 1")
        if num_kv_heads < 1 or head_dim < 1:
            raise ValueError("num_kv_heads and head_dim must be >= 1")
        if dtype not in rt.KV_DTYPE_CODE:
            raise ValueError(f"PagedKVCache: unsupported dtype {dtype}")
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        if dev.type != "cuda":
            raise RuntimeError("PagedKVCache (llmopt_b200) lives in GPU memory: pass a CUDA device")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.num_layers = num_layers
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.device = dev
        shape = (num_layers, num_blocks, block_size, num_kv_heads, head_dim)
        self.key_cache = torch.zeros(shape, dtype=dtype, device=dev)
        self.value_cache = torch.zeros_like(self.key_cache)
        self.key_scale = self.value_scale = None
        if self.is_fp8:
            if head_dim > 256:
                raise ValueError("float8 caches support head_dim <= 256")
            sshape = (num_layers, num_blocks, num_kv_heads, block_size)
            self.key_scale = torch.zeros(sshape, dtype=torch.float32, device=dev)
            self.value_scale = torch.zeros_like(self.key_scale)

    @classmethod
    def from_storage(cls, key_cache: torch.Tensor, value_cache: torch.Tensor,
                     key_scale: torch.Tensor | None = None,
                     value_scale: torch.Tensor | None = None) -> "PagedKVCache":
        """A cache over existing storage (no copy): ``key_cache`` / ``value_cache``
        ``[num_layers, num_blocks, block_size, num_kv_heads, head_dim]`` on a CUDA
        device, plus the two fp32 scale arrays for float8_e4m3fn storage."""
        if key_cache.dim() != 5 or value_cache.shape != key_cache.shape:
            raise ValueError("key_cache/value_cache must be [num_layers, num_blocks, block_size, "
                             "num_kv_heads, head_dim] and alike")
        if key_cache.dtype not in rt.KV_DTYPE_CODE:
            raise ValueError(f"PagedKVCache: unsupported dtype {key_cache.dtype}")
        rt.require_cuda(key_cache, "key_cache")
        self = cls.__new__(cls)
        (self.num_layers, self.num_blocks, self.block_size, self.num_kv_heads,
         self.head_dim) = key_cache.shape
        self.dtype = key_cache.dtype
        self.device = key_cache.device
        self.key_cache = key_cache
        self.value_cache = value_cache
        self.key_scale = key_scale if self.is_fp8 else None
        self.value_scale = value_scale if self.is_fp8 else None
        self._check_storage()
        return self

    @property
    def is_fp8(self) -> bool:
        """e4m3 codes with per-row fp32 scales (``key_scale`` / ``value_scale``)."""
        return self.dtype == torch.float8_e4m3fn

    # -- helpers -----------------------------------------------------------------
    def _layer(self, layer_idx: int) -> int:
        if not -self.num_layers <= layer_idx < self.num_layers:
            raise IndexError(f"layer_idx {layer_idx} out of range for {self.num_layers} layers")
        return layer_idx % self.num_layers

    def _pool_args(self, layer: int):
        return (self.key_cache.data_ptr(), self.value_cache.data_ptr(),
                rt.KV_DTYPE_CODE[self.dtype], self.num_layers, self.num_blocks, self.block_size,
                self.num_kv_heads, self.head_dim, layer)

    def _scaled_pool_args(self, layer: int):
        """The caches, their dtype and the two scale arrays, then the shape."""
        base = self._pool_args(layer)
        return base[:3] + (self.key_scale.data_ptr(), self.value_scale.data_ptr()) + base[3:]

    def _check_storage(self) -> None:
        # The public attributes may be reassigned by callers (benchmarks do); the
        # kernels need the reference layout, contiguous.
        for t in (self.key_cache, self.value_cache):
            if not t.is_contiguous() or t.dtype != self.dtype or t.device != self.device:
                raise ValueError("key_cache/value_cache must stay contiguous, with the cache dtype/device")
        if self.is_fp8:
            shape = (self.num_layers, self.num_blocks, self.num_kv_heads, self.block_size)
            for t in (self.key_scale, self.value_scale):
                if (t is None or not t.is_contiguous() or t.dtype != torch.float32
                        or t.device != self.device or tuple(t.shape) != shape):
                    raise ValueError(f"key_scale/value_scale must stay contiguous fp32 {shape}")

    def _rows(self, x: torch.Tensor, what: str) -> torch.Tensor:
        """Activations may come from anywhere; the kernels read them on our device."""
        if x.device != self.device:
            x = x.to(self.device)
        if x.dtype not in rt.DTYPE_CODE:
            x = x.to(torch.float32)
        if x.stride(-1) != 1:
            x = x.contiguous()
        return x

    # -- reference API -----------------------------------------------------------
    def write(self, layer_idx: int, block_ids: torch.Tensor, token_offsets: torch.Tensor,
              keys: torch.Tensor, values: torch.Tensor) -> None:
        """Scatter ``[seq, q_len, kv_heads, head_dim]`` rows (paged_cache.py:175-232)."""
        seq_len, q_len = keys.shape[0], keys.shape[1]
        if q_len == 0 or seq_len == 0:
            return
        layer = self._layer(layer_idx)
        self._check_storage()
        keys = self._rows(keys, "keys")
        values = self._rows(values, "values")
        if values.dtype != keys.dtype:
            values = values.to(keys.dtype)
        if keys.shape[2:] != (self.num_kv_heads, self.head_dim) or values.shape != keys.shape:
            raise ValueError(f"keys/values must be [seq, q_len, {self.num_kv_heads}, {self.head_dim}]")
        table, t64 = rt.index_tensor(block_ids, self.device, "block_ids")
        offs, o64 = rt.index_tensor(token_offsets, self.device, "token_offsets")
        if table.dim() != 2 or table.shape[0] < seq_len or offs.shape[0] < seq_len:
            raise IndexError("block_ids/token_offsets have fewer rows than keys")
        err = rt.err_word(self.device)
        L = _lib.lib()
        fn, pool = ((L.llmopt_kv_write_scaled, self._scaled_pool_args(layer)) if self.is_fp8
                    else (L.llmopt_kv_write, self._pool_args(layer)))
        st = fn(
            keys.data_ptr(), values.data_ptr(), rt.DTYPE_CODE[keys.dtype],
            keys.stride(0), keys.stride(1), keys.stride(2),
            values.stride(0), values.stride(1), values.stride(2),
            *pool,
            table.data_ptr(), t64, table.shape[1], table.stride(0),
            offs.data_ptr(), o64, seq_len, q_len, err.data_ptr(), rt.stream_handle(self.device))
        _lib.check(st, "PagedKVCache.write")
        if rt.CHECK:
            rt.raise_on_device_errors(self.device, "PagedKVCache.write")

    def write_decode(self, layer_idx: int, block_ids: torch.Tensor, token_offsets: torch.Tensor,
                     keys: torch.Tensor, values: torch.Tensor) -> None:
        """Single-token append of ``[seq, kv_heads, head_dim]`` (paged_cache.py:234-261)."""
        seq_len = keys.shape[0]
        if seq_len == 0:
            return
        self._check_storage()
        keys = self._rows(keys, "keys")
        values = self._rows(values, "values")
        if values.dtype != keys.dtype:
            values = values.to(keys.dtype)
        if keys.shape[1:] != (self.num_kv_heads, self.head_dim) or values.shape != keys.shape:
            raise ValueError(f"keys/values must be [seq, {self.num_kv_heads}, {self.head_dim}]")
        layer = self._layer(layer_idx)
        table, t64 = rt.index_tensor(block_ids, self.device, "block_ids")
        offs, o64 = rt.index_tensor(token_offsets, self.device, "token_offsets")
        if table.dim() != 2 or table.shape[0] < seq_len or offs.shape[0] < seq_len:
            raise IndexError("block_ids/token_offsets have fewer rows than keys")
        err = rt.err_word(self.device)
        L = _lib.lib()
        fn, pool = ((L.llmopt_kv_write_decode_scaled, self._scaled_pool_args(layer))
                    if self.is_fp8 else (L.llmopt_kv_write_decode, self._pool_args(layer)))
        st = fn(
            keys.data_ptr(), values.data_ptr(), rt.DTYPE_CODE[keys.dtype],
            keys.stride(0), keys.stride(1), values.stride(0), values.stride(1),
            *pool,
            table.data_ptr(), t64, table.shape[1], table.stride(0),
            offs.data_ptr(), o64, seq_len, err.data_ptr(), rt.stream_handle(self.device))
        _lib.check(st, "PagedKVCache.write_decode")
        if rt.CHECK:
            rt.raise_on_device_errors(self.device, "PagedKVCache.write_decode")

    def gather(self, layer_idx: int, block_ids: torch.Tensor, context_lens: torch.Tensor):
        """Padded ``(keys, values, valid)`` for a ragged batch (paged_cache.py:263-312)."""
        seq_len = block_ids.shape[0]
        layer = self._layer(layer_idx)
        self._check_storage()
        ctx, c64 = rt.index_tensor(context_lens, self.device, "context_lens")
        if ctx.dim() != 1 or ctx.shape[0] < seq_len:
            raise IndexError("context_lens has fewer entries than block_ids rows")
        max_len = int(ctx.max().item()) if seq_len else 0
        head = (self.num_kv_heads, self.head_dim)
        out_dtype = torch.float32 if self.is_fp8 else self.dtype
        if max_len <= 0:
            empty = torch.zeros((seq_len, 0, *head), dtype=out_dtype, device=self.device)
            return empty, empty.clone(), torch.zeros((seq_len, 0), dtype=torch.bool,
                                                     device=self.device)
        table, t64 = rt.index_tensor(block_ids, self.device, "block_ids")
        if max_len > table.shape[1] * self.block_size:
            raise IndexError("context_lens exceed the block table width")
        keys = torch.empty((seq_len, max_len, *head), dtype=out_dtype, device=self.device)
        values = torch.empty_like(keys)
        valid = torch.empty((seq_len, max_len), dtype=torch.uint8, device=self.device)
        err = rt.err_word(self.device)
        L = _lib.lib()
        fn, pool = ((L.llmopt_paged_gather_scaled, self._scaled_pool_args(layer)) if self.is_fp8
                    else (L.llmopt_paged_gather, self._pool_args(layer)))
        st = fn(
            *pool, table.data_ptr(), t64, table.shape[1], table.stride(0),
            ctx.data_ptr(), c64, seq_len, max_len, keys.data_ptr(), values.data_ptr(),
            valid.data_ptr(), err.data_ptr(), rt.stream_handle(self.device))
        _lib.check(st, "PagedKVCache.gather")
        if rt.CHECK:
            rt.raise_on_device_errors(self.device, "PagedKVCache.gather")
        return keys, values, valid.bool()

    def memory_bytes(self) -> int:
        n = (self.key_cache.numel() * self.key_cache.element_size()
             + self.value_cache.numel() * self.value_cache.element_size())
        if self.is_fp8:
            n += 4 * (self.key_scale.numel() + self.value_scale.numel())
        return n

    def reset(self) -> None:
        self.key_cache.zero_()
        self.value_cache.zero_()
        if self.is_fp8:
            self.key_scale.zero_()
            self.value_scale.zero_()

    def __repr__(self) -> str:
        gib = self.memory_bytes() / float(1 << 30)
        return (f"PagedKVCache(layers={self.num_layers}, blocks={self.num_blocks}, "
                f"block_size={self.block_size}, kv_heads={self.num_kv_heads}, "
                f"head_dim={self.head_dim}, dtype={self.dtype}, size={gib:.2f} GiB, "
                f"device={self.device}, backend=llmopt_b200)")
