"""Python decoder surface over the C ABI.

Mirrors the reference's wrapper classes:
  * ``A10Int8MegakernelDecoder`` -- same constructor arguments and methods as the
    pybind class of bench_int8.py:119-255 (``decode_step``, ``reset``,
    ``position``);
  * ``A10MegakernelDecoder`` -- the BF16 class of a10_decode.py:87-261;
  * ``A10Decoder`` -- the user-facing class of a10_decode.py:35-393 with
    ``.decoder``, ``reset()`` and ``generate()``.
Differences, all additive: constructor arguments are validated (device, dtype,
shape, contiguity); ``decode_step`` raises on an out-of-range token or position
and on a device-side error instead of returning garbage; ``decode_steps`` runs N
greedy steps with on-device token feedback and no host sync.
"""
import ctypes

import torch

from . import _lib
from .config import (CFG, HEAD_DIM, HIDDEN_SIZE, INTERMEDIATE_SIZE, KV_SIZE, MAX_SEQ_LEN, NUM_KV_HEADS,
                     NUM_LAYERS, Q_SIZE, VOCAB_SIZE)
from .quant import quantize_state
from .rope import make_rope

_LAYER_SHAPES = (
    ((HIDDEN_SIZE,), "input_layernorm"), ((Q_SIZE, HIDDEN_SIZE), "q_proj"), ((KV_SIZE, HIDDEN_SIZE), "k_proj"),
    ((KV_SIZE, HIDDEN_SIZE), "v_proj"), ((HEAD_DIM,), "q_norm"), ((HEAD_DIM,), "k_norm"),
    ((HIDDEN_SIZE, Q_SIZE), "o_proj"), ((HIDDEN_SIZE,), "post_attention_layernorm"),
    ((INTERMEDIATE_SIZE, HIDDEN_SIZE), "gate_proj"), ((INTERMEDIATE_SIZE, HIDDEN_SIZE), "up_proj"),
    ((HIDDEN_SIZE, INTERMEDIATE_SIZE), "down_proj"),
)
_SCALE_ROWS = (Q_SIZE, KV_SIZE, KV_SIZE, HIDDEN_SIZE, INTERMEDIATE_SIZE, INTERMEDIATE_SIZE, HIDDEN_SIZE)
_PROJ_IDX = (1, 2, 3, 6, 8, 9, 10)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _check_tensor(t, name, dtype, shape, device):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name}: expected a tensor")
    if t.device != device:
        raise ValueError(f"{name}: on {t.device}, expected {device}")
    if t.dtype != dtype:
        raise ValueError(f"{name}: dtype {t.dtype}, expected {dtype}")
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name}: shape {tuple(t.shape)}, expected {tuple(shape)}")
    if not t.is_contiguous():
        raise ValueError(f"{name}: not contiguous")
    if t.data_ptr() % 16:
        raise ValueError(f"{name}: not 16-byte aligned")


class _MegakernelDecoderBase:
    _kind = 0

    def _common_init(self, embed_weight, layer_weights_flat, final_norm_weight, lm_head, cos_table, sin_table,
                     num_layers, max_seq_len, wdtype):
        if num_layers <= 0 or max_seq_len <= 0:
            raise ValueError("num_layers and max_seq_len must be positive")
        dev = embed_weight.device
        if dev.type != "cuda":
            raise ValueError("the decoder needs CUDA tensors (no CPU path in this library)")
        self.device = dev
        self.num_layers_ = int(num_layers)
        self.max_seq_len_ = int(max_seq_len)
        if len(layer_weights_flat) != 11 * num_layers:
            raise ValueError(f"layer_weights_flat: {len(layer_weights_flat)} tensors, expected {11 * num_layers}")
        _check_tensor(embed_weight, "embed_weight", torch.bfloat16, (VOCAB_SIZE, HIDDEN_SIZE), dev)
        _check_tensor(final_norm_weight, "final_norm_weight", torch.bfloat16, (HIDDEN_SIZE,), dev)
        _check_tensor(lm_head, "lm_head", wdtype, (VOCAB_SIZE, HIDDEN_SIZE), dev)
        for nm, t in (("cos_table", cos_table), ("sin_table", sin_table)):
            _check_tensor(t, nm, torch.bfloat16, (t.shape[0], HEAD_DIM), dev)
            if t.shape[0] < max_seq_len:
                raise ValueError(f"{nm}: {t.shape[0]} rows < max_seq_len {max_seq_len}")
        for i, t in enumerate(layer_weights_flat):
            shape, nm = _LAYER_SHAPES[i % 11]
            dt = wdtype if len(shape) == 2 else torch.bfloat16
            _check_tensor(t, f"layer {i // 11} {nm}", dt, shape, dev)
        self._keep = [embed_weight, final_norm_weight, lm_head, cos_table, sin_table, *layer_weights_flat]
        self.layer_weights_flat_ = list(layer_weights_flat)
        self.embed_weight_, self.final_norm_weight_, self.lm_head_weight_ = embed_weight, final_norm_weight, lm_head
        self.cos_table_, self.sin_table_ = cos_table, sin_table
        arr = (_lib.LayerWeights * num_layers)()
        for i in range(num_layers):
            for j, (fname, _) in enumerate(_lib.LayerWeights._fields_):
                setattr(arr[i], fname, layer_weights_flat[i * 11 + j].data_ptr())
        self.d_layer_weights_ = self._to_device_bytes(arr)  # reference (dense-row) layout
        # Padded copy of every weight matrix (row stride = row bytes + ROW_PAD): the
        # kernel then streams a run of rows with one bulk copy.  Built once here.
        self._pad_keep = []
        parr = (_lib.LayerWeights * num_layers)()
        for i in range(num_layers):
            for j, (fname, _) in enumerate(_lib.LayerWeights._fields_):
                t = layer_weights_flat[i * 11 + j]
                tp = self._padded(t) if t.dim() == 2 else t
                setattr(parr[i], fname, tp.data_ptr())
        self.d_layer_weights_pad_ = self._to_device_bytes(parr)
        self.lm_head_pad_ = self._padded(lm_head)
        shape = (num_layers, NUM_KV_HEADS, max_seq_len, HEAD_DIM)
        self.k_cache_ = torch.zeros(shape, dtype=torch.bfloat16, device=dev)
        self.v_cache_ = torch.zeros(shape, dtype=torch.bfloat16, device=dev)
        self.g_normalized_ = torch.empty(HIDDEN_SIZE, dtype=torch.float32, device=dev)
        self.output_token_ = torch.empty(1, dtype=torch.int32, device=dev)
        self.position_ = 0
        self.attn_scale_ = 1.0 / (HEAD_DIM ** 0.5)
        _lib.load()
        # A decode step reads weights and pointer tables before its dependency
        # wait on the previous kernel: finish writing them here.
        torch.cuda.synchronize(dev)

    def _padded(self, t):
        extra = _lib.ROW_PAD // t.element_size()
        p = torch.zeros((t.shape[0], t.shape[1] + extra), dtype=t.dtype, device=t.device)
        p[:, :t.shape[1]] = t
        self._pad_keep.append(p)
        return p

    def _to_device_bytes(self, carr):
        host = torch.frombuffer(bytearray(bytes(carr)), dtype=torch.uint8)
        return host.to(self.device)

    def _make_plan(self):
        """The fixed launch arguments of decode_step, filled once (MQStepPlan)."""
        scale_lm, scales = self._scale_ptrs()
        self._host_token = torch.empty(1, dtype=torch.int32).pin_memory()
        pl = _lib.MQStepPlan()
        pl.weight_kind, pl.num_layers, pl.max_seq_len = self._kind, self.num_layers_, self.max_seq_len_
        pl.row_pad_bytes, pl.attn_scale = _lib.ROW_PAD, self.attn_scale_
        pl.embed_weight = self.embed_weight_.data_ptr()
        pl.layer_weights = self.d_layer_weights_pad_.data_ptr()
        pl.final_norm_weight = self.final_norm_weight_.data_ptr()
        pl.lm_head_weight = self.lm_head_pad_.data_ptr()
        pl.lm_head_scale, pl.scales = scale_lm.value, scales.value
        pl.cos_table, pl.sin_table = self.cos_table_.data_ptr(), self.sin_table_.data_ptr()
        pl.k_cache, pl.v_cache = self.k_cache_.data_ptr(), self.v_cache_.data_ptr()
        pl.g_normalized = self.g_normalized_.data_ptr()
        pl.host_token = self._host_token.data_ptr()
        self._plan = pl
        self._plan_ref = ctypes.byref(pl)
        self._step_out = ctypes.c_int(0)
        self._step_out_ref = ctypes.byref(self._step_out)
        self._step_fn = _lib.load().mq_decode_step_host
        self._dev_index = self.device.index if self.device.index is not None else torch.cuda.current_device()

    # -- reference methods -------------------------------------------------
    def decode_step(self, input_token_id):
        """One greedy step at position(); returns the argmax token (syncs).
        One C call (mq_decode_step_host): launch on the current stream, the kernel
        writes the token into pinned host memory, stream synchronise."""
        tok = int(input_token_id)
        if not 0 <= tok < VOCAB_SIZE:
            raise ValueError(f"token {tok} outside [0, {VOCAB_SIZE})")
        if self.position_ >= self.max_seq_len_:
            raise ValueError(f"KV cache full: position {self.position_} >= max_seq_len {self.max_seq_len_}")
        if getattr(self, "_plan", None) is None:
            self._make_plan()
        if torch.cuda.current_device() != self._dev_index:
            with torch.cuda.device(self.device):
                return self.decode_step(tok)
        rc = self._step_fn(self._plan_ref, tok, self.position_, torch.cuda.current_stream().cuda_stream,
                           self._step_out_ref)
        if rc:
            if rc == -6:
                _lib.raise_device_error("decode_step")
                raise _lib.MQError("decode_step: kernel reported no token")
            _lib.check(rc, "mq_decode_step_host")
        self.position_ += 1
        return self._step_out.value

    def reset(self):
        self.position_ = 0
        self.k_cache_.zero_()
        self.v_cache_.zero_()

    def position(self):
        return self.position_

    # -- additions ---------------------------------------------------------
    def set_position(self, pos):
        """Move the decode position (e.g. after filling the KV cache externally)."""
        if not 0 <= pos < self.max_seq_len_:
            raise ValueError("position out of range")
        self.position_ = int(pos)

    def decode_steps(self, first_token, num_steps, tokens_out=None, logits=None, layer_hidden=None):
        """Runs num_steps greedy steps from position(); the first input is
        `first_token` (int or a device int32 tensor of one element), each later
        input is the previous output.  Returns the device int32 tensor of
        tokens without synchronising."""
        if num_steps <= 0:
            raise ValueError("num_steps must be positive")
        if self.position_ + num_steps > self.max_seq_len_:
            raise ValueError("decode_steps would run past max_seq_len")
        if isinstance(first_token, torch.Tensor):
            tok_in = first_token
        else:
            if not 0 <= int(first_token) < VOCAB_SIZE:
                raise ValueError("token out of range")
            tok_in = torch.tensor([int(first_token)], dtype=torch.int32, device=self.device)
        if tokens_out is None:
            tokens_out = torch.empty(num_steps, dtype=torch.int32, device=self.device)
        if logits is not None:
            _check_tensor(logits, "logits", torch.float32, (VOCAB_SIZE,), self.device)
        if layer_hidden is not None:
            _check_tensor(layer_hidden, "layer_hidden", torch.float32, (self.num_layers_, HIDDEN_SIZE), self.device)
        self._run(0, tok_in, tokens_out, num_steps, logits, layer_hidden)
        return tokens_out

    def _run(self, tok, tok_dev, tokens_out, num_steps, logits, layer_hidden):
        scale_lm, scales = self._scale_ptrs()
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream(self.device).cuda_stream
            rc = _lib.load().mq_decode_multi(
                self._kind, int(tok), _ptr(tok_dev), _ptr(tokens_out), int(num_steps), _ptr(self.embed_weight_),
                _ptr(self.d_layer_weights_pad_), _ptr(self.final_norm_weight_), _ptr(self.lm_head_pad_), scale_lm,
                scales, _ptr(self.cos_table_), _ptr(self.sin_table_), _ptr(self.k_cache_), _ptr(self.v_cache_),
                _ptr(self.g_normalized_), _ptr(logits), _ptr(layer_hidden), self.num_layers_, self.position_,
                self.max_seq_len_, ctypes.c_float(self.attn_scale_), _lib.ROW_PAD, ctypes.c_void_p(stream))
        _lib.check(rc, "mq_decode_multi")
        self.position_ += num_steps

    def decode_step_reference_abi(self, input_token_id):
        """One step through the reference-signature C entry point
        (launch_a10_int8_decode / launch_a10_decode) on the reference's dense
        weight layout; same result as decode_step."""
        tok = int(input_token_id)
        if not 0 <= tok < VOCAB_SIZE:
            raise ValueError(f"token {tok} outside [0, {VOCAB_SIZE})")
        if self.position_ >= self.max_seq_len_:
            raise ValueError("KV cache full")
        with torch.cuda.device(self.device):
            rc = self._launch(tok, torch.cuda.current_stream(self.device).cuda_stream)
        _lib.check(rc, "decode launch")
        self.position_ += 1
        out = int(self.output_token_.item())
        if out < 0:
            _lib.raise_device_error("decode_step_reference_abi")
        return out

    def check_device(self):
        """Raises if a previous launch recorded a device-side error."""
        _lib.raise_device_error("decoder")

    @property
    def k_cache(self):
        return self.k_cache_

    @property
    def v_cache(self):
        return self.v_cache_

    @property
    def normalized(self):
        return self.g_normalized_


class A10Int8MegakernelDecoder(_MegakernelDecoderBase):
    """INT8 weight-only decoder; constructor of bench_int8.py:121-131."""
    _kind = 0

    def __init__(self, embed_weight, layer_weights_flat, layer_scales_all, lm_head_int8, lm_head_scale,
                 final_norm_weight, cos_table, sin_table, num_layers, max_seq_len):
        self._common_init(embed_weight, layer_weights_flat, final_norm_weight, lm_head_int8, cos_table, sin_table,
                          num_layers, max_seq_len, torch.int8)
        if len(layer_scales_all) != 7 * num_layers:
            raise ValueError(f"layer_scales_all: {len(layer_scales_all)} tensors, expected {7 * num_layers}")
        for i, t in enumerate(layer_scales_all):
            _check_tensor(t, f"layer {i // 7} scale {i % 7}", torch.float32, (_SCALE_ROWS[i % 7],), self.device)
        _check_tensor(lm_head_scale, "lm_head_scale", torch.float32, (VOCAB_SIZE,), self.device)
        self._keep += [lm_head_scale, *layer_scales_all]
        self.lm_head_scale_ = lm_head_scale
        arr = (_lib.ScalePointers * num_layers)()
        for i in range(num_layers):
            for j, (fname, _) in enumerate(_lib.ScalePointers._fields_):
                setattr(arr[i], fname, layer_scales_all[i * 7 + j].data_ptr())
        self.d_layer_scales_ = self._to_device_bytes(arr)

    def prefill(self, token_ids, logits=None):
        """Feeds prompt tokens at positions position() .. position() + n - 1 in
        chunks of up to 64 through the batched tensor-core kernel (one launch per
        chunk, the KV cache filled as by n decode steps) and returns the greedy
        next token (int).  logits (optional): fp32 [n of the last chunk, vocab]."""
        ids = [int(t) for t in token_ids]
        if not ids:
            raise ValueError("empty prompt")
        if any(t < 0 or t >= VOCAB_SIZE for t in ids):
            raise ValueError("token out of range")
        if self.position_ + len(ids) > self.max_seq_len_:
            raise ValueError("prompt exceeds max_seq_len")
        if getattr(self, "_prefiller", None) is None:
            from .batch import Prefiller
            self._prefiller = Prefiller(self)
        out = self._prefiller.run(ids, self.position_, logits)
        self.position_ += len(ids)
        nxt = int(out[-1].item())
        self._prefiller.check_device()
        return nxt

    def _scale_ptrs(self):
        return _ptr(self.lm_head_scale_), _ptr(self.d_layer_scales_)

    def _launch(self, tok, stream):
        n = ctypes.c_void_p(0)
        return _lib.load().launch_a10_int8_decode(
            tok, _ptr(self.output_token_), _ptr(self.embed_weight_), _ptr(self.d_layer_weights_),
            _ptr(self.final_norm_weight_), _ptr(self.lm_head_weight_), _ptr(self.lm_head_scale_),
            _ptr(self.cos_table_), _ptr(self.sin_table_), _ptr(self.k_cache_), _ptr(self.v_cache_),
            n, n, n, n, n, n, n, n, _ptr(self.g_normalized_), n, n,
            self.num_layers_, self.position_, self.position_ + 1, self.max_seq_len_,
            ctypes.c_float(self.attn_scale_), _ptr(self.d_layer_scales_), ctypes.c_void_p(stream))


class A10MegakernelDecoder(_MegakernelDecoderBase):
    """BF16 decoder; constructor of a10_decode.py:89-98."""
    _kind = 1

    def __init__(self, embed_weight, layer_weights_flat, final_norm_weight, lm_head_weight, cos_table, sin_table,
                 num_layers, max_seq_len):
        self._common_init(embed_weight, layer_weights_flat, final_norm_weight, lm_head_weight, cos_table,
                          sin_table, num_layers, max_seq_len, torch.bfloat16)

    def _scale_ptrs(self):
        return ctypes.c_void_p(0), ctypes.c_void_p(0)

    def _launch(self, tok, stream):
        n = ctypes.c_void_p(0)
        return _lib.load().launch_a10_decode(
            tok, _ptr(self.output_token_), _ptr(self.embed_weight_), _ptr(self.d_layer_weights_),
            _ptr(self.final_norm_weight_), _ptr(self.lm_head_weight_), _ptr(self.cos_table_),
            _ptr(self.sin_table_), _ptr(self.k_cache_), _ptr(self.v_cache_),
            n, n, n, n, n, n, n, n, _ptr(self.g_normalized_), n, n,
            self.num_layers_, self.position_, self.position_ + 1, self.max_seq_len_,
            ctypes.c_float(self.attn_scale_), ctypes.c_void_p(stream))


def layer_lists(qstate, num_layers, quantized):
    """Flat tensor lists in the constructor order (bench_int8.py:291-330)."""
    layers, scales = [], []
    for i in range(num_layers):
        p = f"model.layers.{i}"
        names = ("input_layernorm.weight", "self_attn.q_proj.weight", "self_attn.k_proj.weight",
                 "self_attn.v_proj.weight", "self_attn.q_norm.weight", "self_attn.k_norm.weight",
                 "self_attn.o_proj.weight", "post_attention_layernorm.weight", "mlp.gate_proj.weight",
                 "mlp.up_proj.weight", "mlp.down_proj.weight")
        for j, nm in enumerate(names):
            t = qstate[f"{p}.{nm}"]
            layers.append((t[0] if isinstance(t, tuple) else t).contiguous())
        if quantized:
            for j in _PROJ_IDX:
                scales.append(qstate[f"{p}.{names[j]}"][1].contiguous())
    return layers, scales


class A10Decoder:
    """User-facing decoder (a10_decode.py:35-393).

    ``state`` is an HF-named bf16 state dict (e.g. from
    ``synth.make_synthetic_state`` or a real checkpoint's ``state_dict()``);
    ``quantized=True`` builds the INT8 decoder, else the BF16 one.
    ``generate`` takes token ids (and an optional tokenizer for text in/out).
    ``quantized_state`` (INT8 only) is an already quantized state (quantize_state's
    output, e.g. from checkpoint.load_quantized): startup quantization is skipped.
    ``from_pretrained`` builds one from a checkpoint directory.
    """

    def __init__(self, state, quantized=True, max_seq_len=MAX_SEQ_LEN, num_layers=NUM_LAYERS, device="cuda",
                 tokenizer=None, quantized_state=None):
        import os
        if isinstance(state, (str, os.PathLike)):
            # The reference's constructor shape A10Decoder(model_path, max_seq_len)
            # (a10_decode.py:35-36): a checkpoint directory, and an int second
            # positional argument is the sequence limit.
            if not isinstance(quantized, bool):
                max_seq_len, quantized = int(quantized), True
            from . import checkpoint as ck
            path = os.fspath(state)
            if tokenizer is None and (os.path.exists(os.path.join(path, "tokenizer.json")) or
                                      os.path.exists(os.path.join(path, "tokenizer_config.json"))):
                from transformers import AutoTokenizer
                tokenizer = AutoTokenizer.from_pretrained(path, local_files_only=True)
            state = ck.load_state(path, num_layers=num_layers)
        self.device = torch.device(device)
        self.max_seq_len = max_seq_len
        self.tokenizer = tokenizer
        cos, sin = make_rope(max_seq_len, HEAD_DIM, device=self.device, theta=CFG.rope_theta)
        if quantized:
            if quantized_state is not None:
                q = {k: (v[0].to(self.device), v[1].to(self.device)) if isinstance(v, tuple) else v.to(self.device)
                     for k, v in quantized_state.items()}
            else:
                q = quantize_state(state, num_layers=num_layers, device=self.device)
            self.quantized_state = q
            layers, scales = layer_lists(q, num_layers, True)
            lm_q, lm_s = q["lm_head.weight"]
            self.decoder = A10Int8MegakernelDecoder(q["model.embed_tokens.weight"], layers, scales, lm_q, lm_s,
                                                    q["model.norm.weight"], cos, sin, num_layers, max_seq_len)
        else:
            st = {k: v.to(self.device) for k, v in state.items()}
            layers, _ = layer_lists(st, num_layers, False)
            lm = st.get("lm_head.weight", st["model.embed_tokens.weight"])
            self.decoder = A10MegakernelDecoder(st["model.embed_tokens.weight"], layers, st["model.norm.weight"],
                                                lm, cos, sin, num_layers, max_seq_len)

    @classmethod
    def from_pretrained(cls, path, quantized=True, max_seq_len=MAX_SEQ_LEN, num_layers=NUM_LAYERS, device="cuda",
                        tokenizer=True, quantized_path=None):
        """Decoder from an HF Qwen3 checkpoint directory (safetensors).  tokenizer=True
        loads the directory's tokenizer with transformers (local files only) when
        present.  quantized_path: a file written by checkpoint.save_quantized; used
        instead of quantizing when it exists, written after quantizing when not."""
        import os
        from . import checkpoint as ck
        tok = None
        if tokenizer is True:
            if os.path.exists(os.path.join(path, "tokenizer.json")) or os.path.exists(os.path.join(path, "tokenizer_config.json")):
                from transformers import AutoTokenizer
                tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
        elif tokenizer:
            tok = tokenizer
        if quantized and quantized_path and os.path.exists(quantized_path):
            q, n = ck.load_quantized(quantized_path)
            if n != num_layers:
                raise ValueError(f"{quantized_path} holds {n} layers, not {num_layers}")
            return cls(None, True, max_seq_len, num_layers, device, tok, quantized_state=q)
        state = ck.load_state(path, num_layers=num_layers)
        dec = cls(state, quantized, max_seq_len, num_layers, device, tok)
        if quantized and quantized_path:
            ck.save_quantized(dec.quantized_state, quantized_path, num_layers=num_layers)
        return dec

    def reset(self):
        self.decoder.reset()

    def stream(self, prompt, max_new_tokens=128, eos_token_id=None):
        """Like generate, but yields each new token id as soon as it is decoded (the
        decoded text piece instead when a tokenizer was given), for streaming chat
        front ends (the reference's a10_chat.py prints tokens as they come)."""
        ids = self.tokenizer.encode(prompt) if isinstance(prompt, str) else list(prompt)
        if not ids:
            raise ValueError("empty prompt")
        self.reset()
        nxt = self.decoder.prefill(ids) if hasattr(self.decoder, "prefill") else None
        if nxt is None:
            for t in ids:
                nxt = self.decoder.decode_step(t)
        for i in range(max_new_tokens):
            yield self.tokenizer.decode([nxt]) if self.tokenizer is not None else nxt
            if eos_token_id is not None and nxt == eos_token_id:
                return
            if i + 1 == max_new_tokens or self.decoder.position() >= self.max_seq_len:
                return
            nxt = self.decoder.decode_step(nxt)

    def generate(self, prompt, max_new_tokens=128, eos_token_id=None):
        """Greedy generation.  `prompt` is a list of token ids, or a string when a
        tokenizer was given.  INT8: the prompt goes through the chunked prefill
        (64 tokens per launch); BF16: one token per step, as in the reference
        (a10_decode.py:366-369).  Returns the generated id list (or
        text with a tokenizer)."""
        ids = self.tokenizer.encode(prompt) if isinstance(prompt, str) else list(prompt)
        if not ids:
            raise ValueError("empty prompt")
        self.reset()
        if hasattr(self.decoder, "prefill"):   # INT8: chunked prefill on the tensor cores
            nxt = self.decoder.prefill(ids)
        else:
            nxt = None
            for t in ids:
                nxt = self.decoder.decode_step(t)
        out = list(ids)
        for _ in range(max_new_tokens):
            out.append(nxt)
            if eos_token_id is not None and nxt == eos_token_id:
                break
            if self.decoder.position() >= self.max_seq_len:
                break
            nxt = self.decoder.decode_step(nxt)
        return self.tokenizer.decode(out) if self.tokenizer is not None else out
