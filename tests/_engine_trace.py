"""Replay of the reference engine's recorded calls into the paged-KV hot path.

``tests/golden/engine_trace.npz`` (written by ``make_golden.py --only=engine``)
holds, for each of the reference's own engine-correctness scenarios, every
forward call ``ModelRunner.execute`` made (src/llmopt/engine/model_runner.py:92-113):
the input ids and positions, the int32 block table ``_finalize`` built from
the ``BlockPool`` / ``PrefixCache`` chains (:203-230), post-write context
lengths, write offsets and ``q_len``, together with the reference's
last-position logits.  The model weights and the tokens of the reference's
engine and of its stateless ``greedy_reference`` are stored with them.

The reference's code cannot be imported where the GPU tests run, so the tiny
decoder's forward is restated here (fp32, as the engine runs it):

* ``DecoderOnlyModel.forward`` (src/llmopt/model/modeling.py:88-131): embedding,
  the decoder layers, final ``RMSNorm``, ``lm_head``;
* ``DecoderLayer.forward`` (src/llmopt/model/layers.py:176-195): pre-norm
  attention and SwiGLU MLP, both residual;
* ``RMSNorm`` (layers.py:27-31) and ``SwiGLUMLP`` (layers.py:43-44);
* ``PagedAttentionLayer.forward`` (layers.py:79-140): projections, rotary by
  ``apply_rotary_pos_emb`` over the ``RotaryEmbedding`` tables
  (src/llmopt/model/rotary.py:23-46, 64-77), K/V handed to the cache as
  ``[seq, q_len, kv_heads, head_dim]``, ``write_decode`` for ``q_len == 1`` and
  ``write`` otherwise, then ``attn.forward`` -- the calls this package replaces.

The replay is teacher-forced: each call feeds the recorded input ids, so every
call's logits can be compared with the reference's, whatever the earlier
calls' rounding.  A backend supplies the cache and attention:
``OracleBackend`` (numpy restatement, CPU) or ``CudaBackend`` (this package's
``PagedKVCache`` / ``PagedAttention`` on the GPU).
"""

from __future__ import annotations

import json
import os

import numpy as np
import torch

TRACE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "engine_trace.npz")


def load_trace():
    return np.load(TRACE, allow_pickle=False)


def case_names(z) -> list[str]:
    return sorted({k.split(".", 1)[0] for k in z.files if k.endswith(".meta")})


def case_meta(z, name: str) -> dict:
    return json.loads(str(z[f"{name}.meta"]))


def weights(z, meta: dict, device) -> dict:
    pre = meta["weights"] + "."
    return {k[len(pre):]: torch.from_numpy(z[k]).to(device) for k in z.files if k.startswith(pre)}


def calls(z, name: str):
    """Yields one dict per recorded forward call, in order."""
    info = z[f"{name}.calls"]
    ids, pos = z[f"{name}.input_ids"], z[f"{name}.positions"]
    tabs, ctx, offs = z[f"{name}.tables"], z[f"{name}.context_lens"], z[f"{name}.token_offsets"]
    logits = z[f"{name}.logits"]
    io = to = so = 0
    for n_seq, q_len, width in info:
        n_seq, q_len, width = int(n_seq), int(q_len), int(width)
        n_tok = n_seq * q_len
        yield dict(input_ids=ids[io:io + n_tok], positions=pos[io:io + n_tok], q_len=q_len,
                   block_ids=tabs[to:to + n_seq * width].reshape(n_seq, width),
                   context_lens=ctx[so:so + n_seq], token_offsets=offs[so:so + n_seq],
                   logits=logits[so:so + n_seq])
        io += n_tok
        to += n_seq * width
        so += n_seq


def rotary_tables(meta: dict):
    """cos/sin tables built exactly as RotaryEmbedding.__init__ (rotary.py:64-77), on CPU."""
    d, base, n = meta["head_dim"], meta["rope_theta"], meta["max_position_embeddings"]
    inv_freq = 1.0 / (base ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
    freqs = torch.outer(torch.arange(n, dtype=torch.float32), inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos(), emb.sin()


def _rms_norm(x, w, eps):
    x32 = x.to(torch.float32)
    normed = x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps)
    return (normed * w.to(torch.float32)).to(x.dtype)


def _rotate_half(x):
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def forward(meta: dict, w: dict, cos_t, sin_t, backend, call: dict, device) -> torch.Tensor:
    """Last-position logits ``[seq, vocab]`` of one recorded call (fp32)."""
    H, KVH, D, eps = meta["heads"], meta["kv_heads"], meta["head_dim"], meta["rms_norm_eps"]
    q_len = call["q_len"]
    ids = torch.from_numpy(call["input_ids"]).to(device)
    positions = torch.from_numpy(call["positions"]).to(device)
    total = ids.shape[0]
    seq = total // max(1, q_len)
    hidden = w["embed_tokens.weight"][ids]
    cos = cos_t[positions].view(seq, q_len, D).unsqueeze(1)
    sin = sin_t[positions].view(seq, q_len, D).unsqueeze(1)
    for li in range(meta["layers"]):
        p = f"layers.{li}."
        residual = hidden
        h = _rms_norm(hidden, w[p + "input_layernorm.weight"], eps)
        q = (h @ w[p + "self_attn.q_proj.weight"].T).view(seq, q_len, H, D).permute(0, 2, 1, 3)
        k = (h @ w[p + "self_attn.k_proj.weight"].T).view(seq, q_len, KVH, D).permute(0, 2, 1, 3)
        v = (h @ w[p + "self_attn.v_proj.weight"].T).view(seq, q_len, KVH, D).permute(0, 2, 1, 3)
        q = q * cos + _rotate_half(q) * sin
        k = k * cos + _rotate_half(k) * sin
        bk = k.permute(0, 2, 1, 3).contiguous()          # [seq, q_len, kv_heads, head_dim]
        bv = v.permute(0, 2, 1, 3).contiguous()
        if q_len == 1:
            backend.write_decode(li, call, bk[:, 0], bv[:, 0])
        else:
            backend.write(li, call, bk, bv)
        attn = backend.attention(li, call, q)             # [seq, heads, q_len, head_dim]
        attn = attn.to(q.dtype).permute(0, 2, 1, 3).reshape(total, H * D)
        hidden = residual + attn @ w[p + "self_attn.o_proj.weight"].T
        residual = hidden
        h = _rms_norm(hidden, w[p + "post_attention_layernorm.weight"], eps)
        gate = torch.nn.functional.silu(h @ w[p + "mlp.gate_proj.weight"].T)
        hidden = residual + (gate * (h @ w[p + "mlp.up_proj.weight"].T)) @ w[p + "mlp.down_proj.weight"].T
    hidden = _rms_norm(hidden, w["norm.weight"], eps)
    logits = (hidden @ w["lm_head.weight"].T).view(seq, q_len, -1)
    return logits[:, -1, :]


class OracleBackend:
    """The numpy oracle (CPU): bf16 cache bits, fp32 attention arithmetic."""

    def __init__(self, meta: dict):
        from oracle import paged_oracle as po

        self.po = po
        self.kind = {"bfloat16": "bf16", "float16": "f16", "float32": "f32"}[meta["cache_dtype"]]
        shape = (meta["layers"], meta["num_blocks"], meta["block_size"], meta["kv_heads"],
                 meta["head_dim"])
        zero = po.from_f32(np.zeros(shape, dtype=np.float32), self.kind)
        self.kc, self.vc = zero.copy(), zero.copy()
        self.meta = meta

    def write(self, layer, call, k, v):
        self.po.write(self.kc, self.vc, self.kind, layer, call["block_ids"].astype(np.int64),
                      call["token_offsets"], k.numpy(), v.numpy(), "f32")

    def write_decode(self, layer, call, k, v):
        self.po.write_decode(self.kc, self.vc, self.kind, layer,
                             call["block_ids"].astype(np.int64), call["token_offsets"],
                             k.numpy(), v.numpy(), "f32")

    def attention(self, layer, call, q):
        out, _ = self.po.paged_attention(q.numpy().astype(np.float32), "f32", self.kc, self.vc,
                                         self.kind, layer, call["block_ids"].astype(np.int64),
                                         call["context_lens"], self.meta["heads"],
                                         self.meta["kv_heads"], q_len=call["q_len"],
                                         acc=np.float64)
        return torch.from_numpy(out.astype(np.float32))


class CudaBackend:
    """This package's PagedKVCache / PagedAttention on the GPU, called with the
    arguments PagedAttentionLayer.forward passes (layers.py:123-140)."""

    def __init__(self, meta: dict, device, pkg):
        dt = {"bfloat16": torch.bfloat16, "float16": torch.float16,
              "float32": torch.float32}[meta["cache_dtype"]]
        self.cache = pkg.PagedKVCache(meta["layers"], meta["num_blocks"], meta["block_size"],
                                      meta["kv_heads"], meta["head_dim"], dtype=dt,
                                      device=device)
        # The reference layer always builds its attention with block_size=16
        # (layers.py:71-77); the cache's own block size is what addresses it.
        cfg = pkg.PagedAttentionConfig(block_size=16)
        self.attn = pkg.PagedAttention(meta["heads"], meta["kv_heads"], meta["head_dim"],
                                       config=cfg)
        self.device = device

    def _meta(self, call):
        d = self.device
        return (torch.from_numpy(call["block_ids"]).to(d),            # int32, as _finalize
                torch.from_numpy(call["token_offsets"]).to(d),
                torch.from_numpy(call["context_lens"]).to(d))

    def write(self, layer, call, k, v):
        table, offs, _ = self._meta(call)
        self.cache.write(layer, table, offs, k, v)

    def write_decode(self, layer, call, k, v):
        table, offs, _ = self._meta(call)
        self.cache.write_decode(layer, table, offs, k, v)

    def attention(self, layer, call, q):
        table, _, ctx = self._meta(call)
        return self.attn.forward(q, self.cache, layer, table, ctx, call["q_len"])


class LockstepBackend:
    """Runs ``CudaBackend`` and ``OracleBackend`` side by side on identical inputs.

    The oracle receives the GPU-computed K/V and query (copied to the host), so
    each attention output of the GPU path is compared with the oracle's on the
    same bytes; ``check_attention(ours, want, layer)`` does the comparison.  The
    GPU result is what the replayed model continues with.
    """

    def __init__(self, cuda_backend: CudaBackend, oracle_backend: OracleBackend,
                 check_attention):
        self.gpu, self.ref, self.check = cuda_backend, oracle_backend, check_attention

    def write(self, layer, call, k, v):
        self.gpu.write(layer, call, k, v)
        self.ref.write(layer, call, k.float().cpu(), v.float().cpu())

    def write_decode(self, layer, call, k, v):
        self.gpu.write_decode(layer, call, k, v)
        self.ref.write_decode(layer, call, k.float().cpu(), v.float().cpu())

    def attention(self, layer, call, q):
        ours = self.gpu.attention(layer, call, q)
        want = self.ref.attention(layer, call, q.float().cpu())
        self.check(ours.float().cpu().numpy(), want.numpy(), layer)
        return ours


def replay(z, name: str, backend, device, check) -> dict:
    """Replays case ``name`` through ``backend``; ``check(ours, ref_logits, call_index)``
    is called per call.  Returns the per-call last-position argmaxes."""
    meta = case_meta(z, name)
    w = weights(z, meta, device)
    cos_t, sin_t = rotary_tables(meta)
    cos_t, sin_t = cos_t.to(device), sin_t.to(device)
    picks = []
    for i, call in enumerate(calls(z, name)):
        logits = forward(meta, w, cos_t, sin_t, backend, call, device)
        ours = logits.float().cpu().numpy()
        check(ours, call["logits"], i)
        picks.append(ours.argmax(-1))
    return {"meta": meta, "argmax": picks}


def margin_ok(ref_logits: np.ndarray, threshold: float) -> np.ndarray:
    """Rows whose reference top-two logits differ by more than ``threshold``."""
    top2 = np.sort(ref_logits, axis=-1)[:, -2:]
    return (top2[:, 1] - top2[:, 0]) > threshold
