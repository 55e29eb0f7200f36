"""``PagedAttention`` backed by the B200 kernels (drop-in for ``llmopt.attention``).

Mirrors ``src/llmopt/attention/paged_attention.py``: the same
``PagedAttentionConfig`` fields and validation (:58-72), the same
``PagedAttention(num_heads, num_kv_heads, head_dim, scale, config, backend)``
constructor and ``ValueError`` (:127-144), the same
``forward(query, cache, layer_idx, block_ids, context_lens, query_lens)``
contract (:146-187), and ``merge_states`` (:30-55).

``forward`` is one split-K attention kernel plus one combine kernel on the
current CUDA stream; nothing is gathered, padded or expanded, and there is no
host synchronisation.  The split of the context is chosen on the device:

* ``config.split_kv=False``: one split per sequence (the reference's dense path);
* ``config.split_kv=True`` (default): a balanced split-K over the whole batch
  sized from the context lengths and the SM count (``split_mode="auto"``), or
  chunks of ``config.split_size`` tokens rounded up to whole blocks
  (``split_mode="fixed"``, the reference's own chunking).

All modes compute the same exact softmax; they differ only in rounding.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from . import _runtime as rt

__all__ = ["AttentionBackend", "PagedAttention", "PagedAttentionConfig", "merge_states"]


@dataclass(slots=True)
class PagedAttentionConfig:
    """Knobs for the paged attention kernel (paged_attention.py:58-72)."""

    block_size: int = 16
    split_kv: bool = True
    split_size: int = 512
    causal: bool = True
    softcap: float = 0.0

    def __post_init__(self) -> None:
        if self.block_size < 1:
            raise ValueError("block_size must be >= 1")
        if self.split_size < 1:
            raise ValueError("split_size must be >= 1")


class AttentionBackend:
    """Backend names accepted by the reference (paged_attention.py:75-112).

    Every valid request resolves to ``"b200"``: the kernels are the backend.
    Unknown names raise ``ValueError`` as in the reference.
    """

    _known = ("auto", "sdpa", "math", "eager", "flash", "flash_attn", "triton", "b200")

    @classmethod
    def detect(cls, requested: str = "auto") -> str:
        if requested not in cls._known:
            raise ValueError(f"unknown attention backend: {requested!r}")
        return "b200"


def _merge_dtype(a: torch.dtype, b: torch.dtype) -> torch.dtype:
    return torch.promote_types(a, b)


def merge_states(output: torch.Tensor, partial: torch.Tensor, prefix_lse: torch.Tensor,
                 suffix_lse: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Combine two partial attention results using log-sum-exp (paged_attention.py:30-55).

    ``output``/``partial`` are ``[..., seq, head_dim]``, the LSEs ``[..., seq]``.
    Result dtypes follow torch's promotion of the reference's expression.
    """
    for t, name in ((output, "output"), (partial, "partial"), (prefix_lse, "prefix_lse"),
                    (suffix_lse, "suffix_lse")):
        rt.require_cuda(t, f"merge_states {name}")
    if output.shape != partial.shape or prefix_lse.shape != suffix_lse.shape:
        raise ValueError("merge_states: partial shapes must match")
    if tuple(output.shape[:-1]) != tuple(prefix_lse.shape):
        raise ValueError("merge_states: lse must be output.shape[:-1]")
    lse_dtype = _merge_dtype(prefix_lse.dtype, suffix_lse.dtype)
    o_dtype = _merge_dtype(_merge_dtype(output.dtype, partial.dtype), lse_dtype)
    o1 = output.to(o_dtype).contiguous()
    o2 = partial.to(o_dtype).contiguous()
    l1 = prefix_lse.to(lse_dtype).contiguous()
    l2 = suffix_lse.to(lse_dtype).contiguous()
    out = torch.empty_like(o1)
    lse = torch.empty_like(l1)
    head_dim = output.shape[-1] if output.dim() else 1
    rows = l1.numel()
    st = _lib.lib().llmopt_merge_states(
        o1.data_ptr(), o2.data_ptr(), l1.data_ptr(), l2.data_ptr(), out.data_ptr(),
        lse.data_ptr(), rows, head_dim, rt.dtype_code(o_dtype, "merge_states"),
        rt.dtype_code(lse_dtype, "merge_states"), rt.stream_handle(o1.device))
    _lib.check(st, "merge_states")
    return out, lse


class PagedAttention:
    """Attention that reads K/V straight out of a paged cache, on B200 kernels.

    Args:
        num_heads: Query head count.
        num_kv_heads: Key/value head count (``num_heads`` must be a multiple).
        head_dim: Per-head dimension (<= 256).
        scale: Softmax scale; defaults to ``1/sqrt(head_dim)``.
        config: Kernel configuration (any object with the
            :class:`PagedAttentionConfig` fields, the reference's included).
        backend: Accepted for compatibility; always resolves to ``"b200"``.
        split_mode: ``"auto"`` (balanced split-K) or ``"fixed"``
            (``config.split_size`` chunks) when ``config.split_kv`` is set.
    """

    def __init__(self, num_heads: int, num_kv_heads: int, head_dim: int,
                 scale: float | None = None, config: PagedAttentionConfig | None = None,
                 backend: str = "auto", split_mode: str = "auto") -> None:
        if num_heads % num_kv_heads != 0:
            raise ValueError("num_heads must be divisible by num_kv_heads")
        if split_mode not in ("auto", "fixed"):
            raise ValueError("split_mode must be 'auto' or 'fixed'")
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.group_size = num_heads // num_kv_heads
        self.scale = scale if scale is not None else head_dim ** -0.5
        self.config = config or PagedAttentionConfig()
        self.backend = AttentionBackend.detect(backend)
        self.split_mode = split_mode

    def _split_tokens(self) -> int:
        if not self.config.split_kv:
            return _lib.SPLIT_NONE
        if self.split_mode == "fixed":
            return int(self.config.split_size)
        return _lib.SPLIT_AUTO

    def forward(self, query: torch.Tensor, cache, layer_idx: int, block_ids: torch.Tensor,
                context_lens: torch.Tensor, query_lens: int | None = None) -> torch.Tensor:
        """``[seq, num_heads, q_len, head_dim]`` attention output (paged_attention.py:146-187).

        ``context_lens`` is the context length after this step's KV was appended;
        query row ``i`` sits at position ``context_lens - q_len + i``.
        """
        return self.forward_with_lse(query, cache, layer_idx, block_ids, context_lens,
                                     query_lens, want_lse=False)[0]

    def forward_with_lse(self, query: torch.Tensor, cache, layer_idx: int,
                         block_ids: torch.Tensor, context_lens: torch.Tensor,
                         query_lens: int | None = None, want_lse: bool = True,
                         out: torch.Tensor | None = None, phases: int = _lib.PHASE_ALL,
                         gather=None):
        """``forward`` plus the natural-log LSE ``[seq, num_heads, q_len]`` (fp32).

        ``out`` may be any ``[seq, num_heads, q_len, head_dim]`` view with a unit
        innermost stride (for example a slice of a larger buffer); the kernel
        writes into it directly.  ``phases`` selects the split-K kernel
        (``PHASE_SPLIT``), the combine (``PHASE_COMBINE``) or both; issuing the two
        halves as two calls with the same arguments equals one full call.
        ``gather`` (used by ``dist.PeerGroup``) makes the combine also deliver
        the output to every rank of a head-sharded group; ``out`` is then the
        caller's ``[seq, num_heads, q_len, head_dim]`` view of this rank's
        slice of the gathered buffer.
        """
        seq_len = query.shape[0]
        q_len = query_lens if query_lens is not None else query.shape[2]
        if q_len == 0:
            empty = torch.zeros((seq_len, self.num_heads, 0, self.head_dim), dtype=query.dtype,
                                device=query.device)
            return empty, (torch.zeros((seq_len, self.num_heads, 0), dtype=torch.float32,
                                       device=query.device) if want_lse else None)
        if query.dim() != 4 or query.shape[1] != self.num_heads or query.shape[3] != self.head_dim:
            raise ValueError(f"query must be [seq, {self.num_heads}, q_len, {self.head_dim}]")
        if query.shape[2] != q_len:
            raise ValueError(f"query_lens={q_len} does not match query.shape[2]={query.shape[2]}")
        if cache.num_kv_heads != self.num_kv_heads or cache.head_dim != self.head_dim:
            raise ValueError("cache head layout does not match this attention layer")
        rt.require_cuda(cache.key_cache, "cache")
        device = cache.key_cache.device
        if hasattr(cache, "_layer"):
            layer = cache._layer(layer_idx)
            cache._check_storage()
        else:
            layer = layer_idx % cache.num_layers
        out_dtype = query.dtype if query.dtype in rt.DTYPE_CODE else torch.float32
        if query.device != device:
            query = query.to(device)
        if q_len * self.group_size > 16 and cache.key_cache.dtype in (torch.bfloat16, torch.float16):
            # Chunked prefill runs on tensor-core tiles whose operands share one
            # 16-bit type: round the query to the cache dtype first, which is what
            # the reference does (q.to(k.dtype), paged_attention.py:242), and hand
            # the tile loader a dense query.
            query = query.to(cache.key_cache.dtype).contiguous()
        if query.dtype not in rt.DTYPE_CODE:
            query = query.to(torch.float32)
        if query.stride(-1) != 1:
            query = query.contiguous()
        table, t64 = rt.index_tensor(block_ids, device, "block_ids")
        ctx, c64 = rt.index_tensor(context_lens, device, "context_lens")
        if table.dim() != 2 or table.shape[0] < seq_len or ctx.shape[0] < seq_len:
            raise ValueError("block_ids must be [seq, max_blocks] and context_lens [seq]")
        if out is None:
            out = torch.empty((seq_len, self.num_heads, q_len, self.head_dim), dtype=out_dtype,
                              device=device)
        elif out.shape != (seq_len, self.num_heads, q_len, self.head_dim) or out.stride(-1) != 1:
            raise ValueError("out must be [seq, num_heads, q_len, head_dim] with unit inner stride")
        lse = (torch.empty((seq_len, self.num_heads, q_len), dtype=torch.float32, device=device)
               if want_lse else None)
        fp8 = cache.key_cache.dtype == torch.float8_e4m3fn
        if fp8 and gather is not None:
            raise ValueError("the peer-transport gather takes 16-bit or fp32 caches; shard an "
                             "e4m3 cache with transport='nccl'")
        kv_code = rt.KV_DTYPE_CODE.get(cache.key_cache.dtype)
        if kv_code is None:
            raise ValueError(f"cache: unsupported dtype {cache.key_cache.dtype}")
        split = self._split_tokens()
        L = _lib.lib()
        nbytes = _ctypes_size_t()
        _lib.check(L.llmopt_paged_attention_workspace_size(
            device.index, seq_len, self.num_heads, self.num_kv_heads, self.head_dim, q_len,
            cache.block_size, table.shape[1], kv_code, split, nbytes), "workspace size")
        ws = rt.workspace(device, nbytes.value)
        err = rt.err_word(device)
        if rt.CHECK and seq_len and int(ctx[:seq_len].max().item()) > table.shape[1] * cache.block_size:
            raise IndexError("context_lens exceed the block table width")
        scales = ()
        if fp8:
            # e4m3 codes + per-row scales (cache.py); the scaled entry point
            scales = (cache.key_scale.data_ptr(), cache.value_scale.data_ptr())
        common = (query.data_ptr(), rt.DTYPE_CODE[query.dtype], query.stride(0),
                  query.stride(1), query.stride(2),
                  cache.key_cache.data_ptr(), cache.value_cache.data_ptr(), kv_code, *scales,
                  cache.num_layers, cache.num_blocks, cache.block_size, cache.num_kv_heads,
                  cache.head_dim, layer,
                  table.data_ptr(), t64, table.shape[1], table.stride(0),
                  ctx.data_ptr(), c64)
        tail = (seq_len, self.num_heads, q_len, float(self.scale), float(self.config.softcap),
                split, ws.data_ptr(), ws.numel(), err.data_ptr(), rt.stream_handle(device),
                int(phases))
        lse_ptr = lse.data_ptr() if lse is not None else None
        if gather is None:
            entry = L.llmopt_paged_attention_scaled if fp8 else L.llmopt_paged_attention_phase
            st = entry(
                *common, out.data_ptr(), rt.dtype_code(out.dtype, "out"), out.stride(0),
                out.stride(1), out.stride(2), lse_ptr, *tail)
        else:
            bufs, flags, world, rank, epoch = gather
            st = L.llmopt_paged_attention_gather(
                *common, bufs, flags, world, rank, epoch, rt.dtype_code(out.dtype, "out"),
                lse_ptr, *tail)
        _lib.check(st, "PagedAttention.forward")
        if rt.CHECK:
            rt.raise_on_device_errors(device, "PagedAttention.forward")
        return out, lse

    __call__ = forward

    def _forward_dense(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                       valid: torch.Tensor, context_lens: torch.Tensor,
                       q_len: int) -> torch.Tensor:
        """Attention over dense K/V with no cache (paged_attention.py:231-250).

        ``PagedAttentionLayer._dense_attention`` (layers.py:144-163) calls this
        for the model's stateless forward (``cache=None``), the path the
        reference's engine tests compare against.  ``k`` / ``v`` are
        ``[seq, kv_heads, ctx, head_dim]``; they are copied once into a
        temporary block pool in ``k``'s dtype, addressed by an identity block
        table, and the paged kernels run over it, so query row ``i`` of sequence
        ``s`` attends to key positions ``<= context_lens[s] - q_len + i`` (the
        causal rule of ``_build_mask``, :212-229).  ``valid`` must hold every
        position below ``context_lens`` (the layer passes it all true): the
        kernels mask positions from ``context_lens`` on, and a hole inside the
        context raises ``ValueError``.
        """
        if k.dim() != 4 or v.shape != k.shape:
            raise ValueError("k and v must be [seq, kv_heads, ctx, head_dim] and alike")
        seq, kvh, ctx, d = k.shape
        rt.require_cuda(k, "k")
        device = k.device
        lens = context_lens.to(device=device, dtype=torch.int64).reshape(-1)
        if lens.numel() < seq:
            raise ValueError("context_lens must have one entry per sequence")
        pos = torch.arange(ctx, device=device)
        inside = pos[None, :] < lens[:seq, None]
        if not bool((valid.to(device)[:seq, :ctx] | ~inside).all()):
            raise ValueError("valid must hold every position below context_lens")
        bs = 16
        nb = max(1, -(-ctx // bs))
        dtype = k.dtype if k.dtype in rt.KV_DTYPE_CODE else torch.float32
        pools = []
        for t in (k, v):
            pool = torch.zeros((1, seq * nb, bs, kvh, d), dtype=dtype, device=device)
            pool.view(seq, nb * bs, kvh, d)[:, :ctx] = t.permute(0, 2, 1, 3)
            pools.append(pool)
        from .cache import PagedKVCache

        cache = PagedKVCache.from_storage(*pools)
        table = torch.arange(seq * nb, dtype=torch.int32, device=device).view(seq, nb)
        return self.forward(q, cache, 0, table, lens[:seq], q_len)

    def __repr__(self) -> str:
        return (f"PagedAttention(heads={self.num_heads}, kv_heads={self.num_kv_heads}, "
                f"head_dim={self.head_dim}, backend={self.backend}, "
                f"split_kv={self.config.split_kv}, split_mode={self.split_mode})")


def _ctypes_size_t():
    import ctypes

    return ctypes.c_size_t(0)
