"""Batched greedy decode: up to 64 independent sequences,
each at its own position with its own KV cache, advance one token per step
while sharing one pass over the INT8 weights (csrc/batch_kernel.cu).

`BatchedDecoder` takes the INT8 weights of an `A10Int8MegakernelDecoder`,
tile-packs every matrix once (`pack_tiles`: the layout the batched kernel's
bulk copies and tensor-core GEMMs read) and owns the per-sequence state: KV
caches [B][L][8][max_seq][128] bf16, the token and position vectors and the
kernel's workspace -- all allocated here with torch, so the C entry point
itself allocates nothing.
"""
import ctypes

import torch

from . import _lib
from .config import HEAD_DIM, NUM_KV_HEADS, VOCAB_SIZE


class MQBatchArgs(ctypes.Structure):
    """Mirror of MQBatchArgs in include/megaqwen_b200.h."""
    _fields_ = [
        ("embed_weight", ctypes.c_void_p), ("layer_weights", ctypes.c_void_p), ("scales", ctypes.c_void_p),
        ("final_norm_weight", ctypes.c_void_p), ("lm_head_weight", ctypes.c_void_p),
        ("lm_head_scale", ctypes.c_void_p), ("cos_table", ctypes.c_void_p), ("sin_table", ctypes.c_void_p),
        ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p), ("tokens", ctypes.c_void_p),
        ("positions", ctypes.c_void_p), ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
        ("logits", ctypes.c_void_p), ("trace", ctypes.c_void_p), ("wait_budget_ns", ctypes.c_ulonglong),
        ("batch", ctypes.c_int),
        ("num_layers", ctypes.c_int), ("max_seq_len", ctypes.c_int), ("attn_scale", ctypes.c_float),
        ("prefill", ctypes.c_int), ("vocab_shards", ctypes.c_int), ("vocab_shard", ctypes.c_int),
        ("keys_out", ctypes.c_void_p),
    ]


def pack_tiles(w, slab_major=False, block_k=64):
    """INT8 [rows, K] (rows % 16 == 0, K % block_k == 0) -> packed copy (same bytes):
    tile-major 16-row x 64-column 1 KB blocks (mq_pack_weight_tiles, the stand-alone
    GEMM) or slab-major 16-row x block_k blocks (mq_pack_weight_slabs: the batched
    decode's projections with block_k 256, its LM head with 64)."""
    if w.dtype != torch.int8 or w.dim() != 2 or not w.is_cuda or not w.is_contiguous():
        raise ValueError("pack_tiles: contiguous CUDA int8 [rows, K] expected")
    out = torch.empty_like(w)
    lib = _lib.load()
    with torch.cuda.device(w.device):
        stream = ctypes.c_void_p(torch.cuda.current_stream(w.device).cuda_stream)
        src, dst = ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(out.data_ptr())
        if slab_major:
            rc = lib.mq_pack_weight_slabs(src, w.shape[0], w.shape[1], w.shape[1], int(block_k), dst, stream)
        else:
            rc = lib.mq_pack_weight_tiles(src, w.shape[0], w.shape[1], w.shape[1], dst, stream)
        _lib.check(rc, "pack_tiles")
    return out


def batch_matmul(w_tiles, scale, x):
    """y[t, m] = scale[m] * sum_k W[m, k] x[t, k] on the batched path's tensor-core GEMM.
    w_tiles: pack_tiles(W) of an int8 [M, K]; scale fp32 [M]; x fp32 [B <= 64, K]."""
    M, K = w_tiles.shape
    B = x.shape[0]
    y = torch.empty((B, M), dtype=torch.float32, device=x.device)
    lib = _lib.load()
    nbytes = ctypes.c_size_t(0)
    _lib.check(lib.mq_batch_matmul_workspace_bytes(K, ctypes.byref(nbytes)), "mq_batch_matmul_workspace_bytes")
    ws = torch.empty(nbytes.value, dtype=torch.uint8, device=x.device)
    xc = x.contiguous()
    with torch.cuda.device(x.device):
        stream = torch.cuda.current_stream(x.device).cuda_stream
        _lib.check(lib.mq_batch_matmul(ctypes.c_void_p(w_tiles.data_ptr()), ctypes.c_void_p(scale.data_ptr()),
                                       ctypes.c_void_p(xc.data_ptr()), ctypes.c_void_p(y.data_ptr()), M, K, B,
                                       ctypes.c_void_p(ws.data_ptr()), nbytes.value, ctypes.c_void_p(stream)),
                   "mq_batch_matmul")
    torch.cuda.synchronize(x.device)
    code, info = ctypes.c_int(0), ctypes.c_int(0)
    _lib.check(lib.mq_batch_status(ctypes.c_void_p(ws.data_ptr()), ctypes.byref(code), ctypes.byref(info)),
               "mq_batch_status")
    if code.value:
        raise _lib.MQError(f"batch_matmul: device error {code.value} at {info.value}")
    return y


def packed_weights(dec):
    """(device LayerWeights table of the slab-packed projections (q|k|v fused, gate/up
    interleaved), slab-packed LM
    head) of an A10Int8MegakernelDecoder, built once and kept on the decoder."""
    pk = getattr(dec, "_packed_", None)
    if pk is None:
        keep = []
        arr = (_lib.LayerWeights * dec.num_layers_)()
        flat = dec.layer_weights_flat_
        names = [f for f, _ in _lib.LayerWeights._fields_]
        for i in range(dec.num_layers_):
            t = {n: flat[i * 11 + j] for j, n in enumerate(names)}
            qkv = pack_tiles(torch.cat([t["q_proj_weight"], t["k_proj_weight"], t["v_proj_weight"]], 0).contiguous(),
                             slab_major=True, block_k=256)
            g, u = t["gate_proj_weight"], t["up_proj_weight"]
            gu = torch.stack([g.view(-1, 16, g.shape[1]), u.view(-1, 16, u.shape[1])], 1).reshape(-1, g.shape[1])
            gu = pack_tiles(gu.contiguous(), slab_major=True, block_k=256)
            o = pack_tiles(t["o_proj_weight"], slab_major=True, block_k=256)
            d = pack_tiles(t["down_proj_weight"], slab_major=True, block_k=256)
            keep += [qkv, gu, o, d]
            packed = {"q_proj_weight": qkv, "k_proj_weight": qkv, "v_proj_weight": qkv, "o_proj_weight": o,
                      "gate_proj_weight": gu, "up_proj_weight": gu, "down_proj_weight": d}
            for n in names:
                setattr(arr[i], n, packed.get(n, t[n]).data_ptr())
        table = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8).to(dec.device)
        lm = pack_tiles(dec.lm_head_weight_, slab_major=True)
        pk = dec._packed_ = (table, lm, keep)
    return pk[0], pk[1]


_SIGN = -(2 ** 63)


def pack_keys(logits, row0=0):
    """Host statement of the kernel's argmax key for fp32 logits [B, n] of vocab rows
    row0 .. row0 + n - 1: (order(logit) << 32 | ~row) with the sign bit flipped, as
    int64 [B] (the max over the rows).  Used to test the shard reduction."""
    u = logits.float().contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    order = torch.where(u >= 2 ** 31, (~u) & 0xFFFFFFFF, u | 2 ** 31)
    rows = torch.arange(row0, row0 + logits.shape[1], dtype=torch.int64)
    k = (order << 32) | ((~rows) & 0xFFFFFFFF)
    return (k ^ _SIGN).max(dim=1).values


def reduce_shard_keys(keys, dist, group=None):
    """Global argmax keys from every rank's vocab-shard keys (int64 max all-reduce, in place)."""
    if dist is not None:
        dist.all_reduce(keys, op=dist.ReduceOp.MAX, group=group)
    return keys


def keys_to_tokens(keys):
    """Token ids (int32) from packed keys: the low 32 bits hold ~row."""
    return ((~(keys ^ _SIGN)) & 0xFFFFFFFF).to(torch.int32)


def _launch(dec, table, lm, kc, vc, tokens, positions, ws, batch, max_seq, num_steps, logits, trace, prefill,
            shards=0, shard=0, keys=None):
    a = MQBatchArgs(dec.embed_weight_.data_ptr(), table.data_ptr(), dec.d_layer_scales_.data_ptr(),
                    dec.final_norm_weight_.data_ptr(), lm.data_ptr(), dec.lm_head_scale_.data_ptr(),
                    dec.cos_table_.data_ptr(), dec.sin_table_.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                    tokens.data_ptr(), positions.data_ptr(), ws.data_ptr(), ws.numel(),
                    logits.data_ptr() if logits is not None else None,
                    trace.data_ptr() if trace is not None else None, 0, batch, dec.num_layers_, max_seq,
                    dec.attn_scale_, int(prefill), int(shards), int(shard),
                    keys.data_ptr() if keys is not None else None)
    with torch.cuda.device(dec.device):
        stream = torch.cuda.current_stream(dec.device).cuda_stream
        rc = _lib.load().mq_batch_decode(ctypes.byref(a), int(num_steps), ctypes.c_void_p(stream))
    _lib.check(rc, "mq_batch_decode")


def _status(ws):
    code, info = ctypes.c_int(0), ctypes.c_int(0)
    _lib.check(_lib.load().mq_batch_status(ctypes.c_void_p(ws.data_ptr()), ctypes.byref(code), ctypes.byref(info)),
               "mq_batch_status")
    return code.value, info.value


class Prefiller:
    """Chunked prefill of one sequence into an A10Int8MegakernelDecoder's own KV
    cache: up to 64 prompt tokens per launch go through the batched tensor-core
    kernel as rows of one sequence (MQBatchArgs.prefill = 1).  Replaces feeding
    the prompt one decode step per token (a10_decode.py:366-369)."""
    CHUNK = 64

    def __init__(self, dec):
        if dec.max_seq_len_ > 32768:
            raise ValueError("prefill needs max_seq_len <= 32768")
        self.dec = dec
        self.table, self.lm = packed_weights(dec)
        dev = dec.device
        self.tokens = torch.zeros(self.CHUNK, dtype=torch.int32, device=dev)
        self.positions = torch.zeros(self.CHUNK, dtype=torch.int32, device=dev)
        nbytes = ctypes.c_size_t(0)
        _lib.check(_lib.load().mq_batch_workspace_bytes(self.CHUNK, ctypes.byref(nbytes)), "mq_batch_workspace_bytes")
        self.workspace = torch.zeros(nbytes.value, dtype=torch.uint8, device=dev)

    def run(self, ids, start, logits=None):
        """Tokens ids at positions start .. start + len(ids) - 1; returns the device
        int32 vector of the last chunk's argmax outputs (its last entry is the
        greedy next token).  logits (optional): fp32 [len(last chunk), vocab]."""
        d = self.dec
        out = None
        for c0 in range(0, len(ids), self.CHUNK):
            chunk = ids[c0:c0 + self.CHUNK]
            n = len(chunk)
            self.tokens[:n].copy_(torch.as_tensor(chunk, dtype=torch.int32))
            self.positions[:n].copy_(torch.arange(start + c0, start + c0 + n, dtype=torch.int32))
            last = c0 + self.CHUNK >= len(ids)
            _launch(d, self.table, self.lm, d.k_cache_, d.v_cache_, self.tokens, self.positions, self.workspace, n,
                    d.max_seq_len_, 1, logits if last else None, None, True)
            out = self.tokens[:n]
        return out

    def check_device(self):
        code, info = _status(self.workspace)
        if code:
            raise _lib.MQError(f"prefill: device error {code} ({_lib.MQ_DEV_ERRORS.get(code, '?')}, at {info})")


class BatchedDecoder:
    MAX_BATCH = 64

    def __init__(self, weights, batch, max_seq_len, vocab_shard=None):
        """weights: an A10Int8MegakernelDecoder (its INT8 matrices are packed here, once per decoder);
        max_seq_len <= 32768 and <= the rows of its RoPE tables.
        vocab_shard: (rank, world, dist, group) to split the LM head over `world`
        ranks that decode the SAME sequences (same tokens and caches on every
        rank): each scores 1/world of the vocabulary and one int64 max all-reduce
        per step picks the global argmax (lowest index on ties)."""
        if not 1 <= batch <= self.MAX_BATCH:
            raise ValueError(f"batch must be in [1, {self.MAX_BATCH}]")
        if not 1 <= max_seq_len <= min(32768, weights.cos_table_.shape[0]):
            raise ValueError("max_seq_len out of range")
        self.w = weights
        self.device = weights.device
        self.vocab_shard = vocab_shard
        self.d_layer_tiles_, self.lm_head_tiles_ = packed_weights(weights)
        self.B, self.L, self.max_seq_len = batch, weights.num_layers_, max_seq_len
        shape = (batch, self.L, NUM_KV_HEADS, max_seq_len, HEAD_DIM)
        self.k_cache = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        self.v_cache = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        self.tokens = torch.zeros(batch, dtype=torch.int32, device=self.device)
        self.positions = torch.zeros(batch, dtype=torch.int32, device=self.device)
        nbytes = ctypes.c_size_t(0)
        _lib.check(_lib.load().mq_batch_workspace_bytes(batch, ctypes.byref(nbytes)), "mq_batch_workspace_bytes")
        self.workspace = torch.zeros(nbytes.value, dtype=torch.uint8, device=self.device)
        self.keys = torch.zeros(batch, dtype=torch.int64, device=self.device)

    def set_state(self, tokens, positions):
        """Input token and position (cache_len = position + 1) of every sequence."""
        t = torch.as_tensor(tokens, dtype=torch.int32).to(self.device)
        p = torch.as_tensor(positions, dtype=torch.int32).to(self.device)
        if t.shape != (self.B,) or p.shape != (self.B,):
            raise ValueError("tokens and positions must have one entry per sequence")
        if int(t.min()) < 0 or int(t.max()) >= VOCAB_SIZE:
            raise ValueError("token out of range")
        if int(p.min()) < 0 or int(p.max()) >= self.max_seq_len:
            raise ValueError("position out of range")
        self.tokens.copy_(t)
        self.positions.copy_(p)

    def step(self, num_steps=1, logits=None, trace=None):
        """Runs num_steps greedy steps for every sequence (on-device token feedback;
        no host sync).  Returns the device token vector (the last step's outputs)."""
        if logits is not None and (logits.dtype != torch.float32 or tuple(logits.shape) != (self.B, VOCAB_SIZE)):
            raise ValueError("logits must be fp32 [batch, vocab]")
        if self.vocab_shard is None:
            _launch(self.w, self.d_layer_tiles_, self.lm_head_tiles_, self.k_cache, self.v_cache, self.tokens,
                    self.positions, self.workspace, self.B, self.max_seq_len, num_steps, logits, trace, False)
            return self.tokens
        rank, world, dist, group = self.vocab_shard
        for _ in range(num_steps):   # one launch + one all-reduce per step
            _launch(self.w, self.d_layer_tiles_, self.lm_head_tiles_, self.k_cache, self.v_cache, self.tokens,
                    self.positions, self.workspace, self.B, self.max_seq_len, 1, None, trace, False,
                    shards=world, shard=rank, keys=self.keys)
            reduce_shard_keys(self.keys, dist if world > 1 else None, group)
            self.tokens.copy_(keys_to_tokens(self.keys))
        return self.tokens

    def status(self):
        return _status(self.workspace)

    def check_device(self):
        code, info = self.status()
        if code:
            raise _lib.MQError(f"batched decode: device error {code} ({_lib.MQ_DEV_ERRORS.get(code, '?')}, at {info})")
