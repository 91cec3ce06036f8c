"""Host mirror of the whole-model greedy decode engines (C ABI tq_gpt2_*,
tq_qwen_*).

Gpt2 stands for the GPT-2 example's model (_example/gpt2/model.go) with
random-init weights: Gpt2(cfg, seed, sigma).generate(prompt, n) runs the
fp32 prefill and the int8 decode steps on the GPU and returns the greedy
token ids (main.go:163-170 at temperature 0). Qwen does the same for the
Qwen2 example (_example/qwen/model.go) with int4 weights, tensor-parallel
over the ranks of a process group (one process per GPU).
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib

GPT2_SMALL = dict(n_layer=12, n_head=12, d=768, ffn=3072, vocab=50257, ctx=1024)


class Gpt2Config(ctypes.Structure):
    _fields_ = [("n_layer", ctypes.c_int), ("n_head", ctypes.c_int), ("d", ctypes.c_int), ("ffn", ctypes.c_int),
                ("vocab", ctypes.c_int), ("ctx", ctypes.c_int)]


def synth_tokens(n: int, vocab: int, seed: int) -> np.ndarray:
    """Seeded uniform token ids in [0, vocab): a stand-in for a tokenized prompt."""
    out = np.empty(n, np.int32)
    _lib.check(_lib.load().tq_synth_tokens(out.ctypes.data_as(ctypes.c_void_p), n, vocab, seed))
    return out


def _checkpoint_tensors(path: str):
    """(name, CUDA tensor in its stored type) for each tensor of a .safetensors
    file or a model.safetensors.index.json, one at a time."""
    from . import safetensors as ST
    src = ST.OpenSharded(path) if path.endswith(".json") else ST.Open(path)
    try:
        for name in src.Names():
            f = src.File(name) if isinstance(src, ST.Shards) else src
            yield name, f.DeviceTensor(name)
    finally:
        src.Close()


def _load_into(fn, handle: int, name: str, t) -> None:
    """tq_*_load_tensor of one CUDA tensor (float32, float16 or bfloat16)."""
    import torch
    kinds = {torch.float32: _lib.TQ_LINEAR_F32, torch.float16: _lib.TQ_LINEAR_F16, torch.bfloat16: _lib.TQ_LINEAR_BF16}
    if t.dtype not in kinds or t.dim() not in (1, 2) or not t.is_contiguous():
        raise ValueError(f"tensai: {name}: a contiguous 1-D or 2-D float32, float16 or bfloat16 tensor is required")
    rows, cols = (1, t.shape[0]) if t.dim() == 1 else (t.shape[0], t.shape[1])
    _lib.check(fn(handle, name.encode(), ctypes.c_void_p(t.data_ptr()), kinds[t.dtype], rows, cols))


class Gpt2:
    """A resident GPT-2 on the current device: random-init weights from a seed,
    or a checkpoint's (from_checkpoint)."""

    def __init__(self, cfg: dict, seed: int, sigma: float = 0.02):
        self.cfg = dict(cfg)
        h = ctypes.c_uint64()
        c = Gpt2Config(**self.cfg)
        _lib.check(_lib.load().tq_gpt2_create(ctypes.byref(c), seed, ctypes.c_float(sigma), ctypes.byref(h)))
        self.handle = h.value
        self.last_times_ms = (0.0, 0.0)

    @classmethod
    def from_checkpoint(cls, cfg: dict, path: str) -> "Gpt2":
        """A GPT-2 with a Hugging Face checkpoint's weights (the example's
        loader, _example/gpt2/model.go:83-131): the tensors go to the GPU in
        their stored type (tq_gpt2_create_empty, tq_gpt2_load_tensor); a
        "transformer." name prefix is dropped, and the attention-mask buffers
        and a tied lm_head.weight are skipped (the head is wte^T)."""
        self = cls.__new__(cls)
        self.cfg = dict(cfg)
        h = ctypes.c_uint64()
        _lib.check(_lib.load().tq_gpt2_create_empty(ctypes.byref(Gpt2Config(**self.cfg)), ctypes.byref(h)))
        self.handle = h.value
        self.last_times_ms = (0.0, 0.0)
        try:
            for name, t in _checkpoint_tensors(path):
                name = name[len("transformer."):] if name.startswith("transformer.") else name
                if name == "lm_head.weight" or name.endswith(".attn.bias") or name.endswith(".attn.masked_bias"):
                    continue
                self.load_tensor(name, t)
        except BaseException:
            self.free()
            raise
        return self

    def load_tensor(self, name: str, t) -> None:
        """One checkpoint tensor (a CUDA tensor as stored) by the example's name."""
        _load_into(_lib.load().tq_gpt2_load_tensor, self.handle, name, t)

    def generate(self, prompt, n: int) -> np.ndarray:
        """Greedy ids of the n tokens after the prompt; last_times_ms holds the
        device time of the prefill and of the decode steps."""
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.empty(n, np.int32)
        t = (ctypes.c_float * 2)()
        _lib.check(_lib.load().tq_gpt2_generate(self.handle, p.ctypes.data_as(ctypes.c_void_p), len(p), n,
                                                out.ctypes.data_as(ctypes.c_void_p), t))
        self.last_times_ms = (t[0], t[1])
        return out

    def set_sampling(self, temp: float, draws=None) -> None:
        """temp <= 0: greedy (the default); temp > 0: generated token k is
        drawn by the sample step with draws[k] (tq_gpt2_set_sampling)."""
        d = np.ascontiguousarray(draws if draws is not None else [], np.float64)
        _lib.check(_lib.load().tq_gpt2_set_sampling(self.handle, float(temp), d.ctypes.data_as(ctypes.c_void_p) if len(d)
                                                    else None, len(d)))

    def free(self) -> None:
        if self.handle:
            _lib.load().tq_gpt2_free(self.handle)
            self.handle = 0

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.free()


# ---------------------------------------------------------------------------
# Qwen2 (int4), tensor parallel
# ---------------------------------------------------------------------------

QWEN_7B = dict(n_layer=28, n_head=28, n_kv=4, d=3584, ffn=18944, vocab=152064, ctx=2560, eps=1e-6, theta=1e6)


def sample(logits, temp: float, u: float) -> int:
    """The examples' sample (_example/gpt2/main.go:78-105) on the GPU
    (tq_sample): greedy at temp <= 0, else a draw from the tempered
    distribution with the caller's uniform u (rng.Float64() in the Go code)."""
    v = np.ascontiguousarray(logits, np.float32)
    tok = ctypes.c_int()
    _lib.check(_lib.load().tq_sample(v.ctypes.data_as(ctypes.c_void_p), len(v), float(temp), float(u),
                                     ctypes.byref(tok)))
    return tok.value


class QwenConfig(ctypes.Structure):
    _fields_ = [("n_layer", ctypes.c_int), ("n_head", ctypes.c_int), ("n_kv", ctypes.c_int), ("d", ctypes.c_int),
                ("ffn", ctypes.c_int), ("vocab", ctypes.c_int), ("ctx", ctypes.c_int), ("eps", ctypes.c_double),
                ("theta", ctypes.c_double)]


def qwen_shard_plan(cfg: dict, world: int, rank: int) -> dict:
    """The slices of the model that rank `rank` of `world` holds, from the
    library (tq_qwen_shard_plan, the rule tq_qwen_create applies): attention
    heads, o_proj rows, MLP columns (gate/up) = down rows, lm-head columns.
    Raises ValueError when the configuration does not split over `world` GPUs."""
    c = QwenConfig(**cfg)
    plan = (ctypes.c_int * 12)()
    L = _lib.load()
    rc = L.tq_qwen_shard_plan(ctypes.byref(c), world, rank, plan)
    if rc != _lib.TQ_OK:
        raise ValueError(L.tq_last_error().decode())
    v = list(plan)
    return dict(q_heads=(v[0], v[1]), kv_heads=(v[2], v[3]), o_rows=(v[4], v[5]), att_dims=(v[6], v[7]),
                ffn=(v[8], v[9]), vocab=(v[10], v[11]))


def nccl_unique_id() -> bytes:
    buf = (ctypes.c_char * 128)()
    _lib.check(_lib.load().tq_nccl_unique_id(buf))
    return bytes(buf)


def broadcast_nccl_id(dist) -> bytes:
    """Rank 0 makes an NCCL unique id; every rank of the process group gets it."""
    obj = [nccl_unique_id() if dist.get_rank() == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    return obj[0]


class Qwen:
    """This rank's shard of a resident Qwen2 (int4) on the current device:
    random-init weights from a seed, or (one GPU) a checkpoint's
    (from_checkpoint). world > 1: every rank builds its shard at the same time
    with the same nccl_id (see broadcast_nccl_id) and calls generate together."""

    def __init__(self, cfg: dict, seed: int, sigma: float = 0.02, rank: int = 0, world: int = 1,
                 nccl_id: bytes | None = None):
        self.cfg = dict(cfg)
        c = QwenConfig(**self.cfg)
        h = ctypes.c_uint64()
        idp = ctypes.create_string_buffer(nccl_id, 128) if nccl_id else None
        _lib.check(_lib.load().tq_qwen_create(ctypes.byref(c), seed, ctypes.c_float(sigma), rank, world, idp,
                                              ctypes.byref(h)))
        self.handle = h.value
        self.last_times_ms = (0.0, 0.0)

    @classmethod
    def from_checkpoint(cls, cfg: dict, path: str) -> "Qwen":
        """A one-GPU model with a Hugging Face Qwen2 checkpoint's weights
        (loadQwen, _example/qwen/model.go:95-177): `path` is a .safetensors
        file or a model.safetensors.index.json. Each tensor goes to the GPU in
        its stored type and is quantized there (tq_qwen_create_empty,
        tq_qwen_load_tensor); a checkpoint without lm_head.weight ties it to
        the embedding."""
        self = cls.__new__(cls)
        self.cfg = dict(cfg)
        c = QwenConfig(**self.cfg)
        h = ctypes.c_uint64()
        _lib.check(_lib.load().tq_qwen_create_empty(ctypes.byref(c), ctypes.byref(h)))
        self.handle = h.value
        self.last_times_ms = (0.0, 0.0)
        try:
            embed, have_head = None, False
            for name, t in _checkpoint_tensors(path):
                if name.endswith("rotary_emb.inv_freq"):
                    continue  # recomputed from theta
                self.load_tensor(name, t)
                have_head = have_head or name == "lm_head.weight"
                if name == "model.embed_tokens.weight":
                    embed = t
            if not have_head and embed is not None:
                self.load_tensor("lm_head.weight", embed)
        except BaseException:
            self.free()
            raise
        return self

    def load_tensor(self, name: str, t) -> None:
        """One checkpoint tensor (a CUDA tensor of float32, float16 or
        bfloat16, in the checkpoint's layout) by its name (tq_qwen_load_tensor)."""
        _load_into(_lib.load().tq_qwen_load_tensor, self.handle, name, t)

    def generate(self, prompt, n: int) -> np.ndarray:
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.empty(n, np.int32)
        t = (ctypes.c_float * 2)()
        _lib.check(_lib.load().tq_qwen_generate(self.handle, p.ctypes.data_as(ctypes.c_void_p), len(p), n,
                                                out.ctypes.data_as(ctypes.c_void_p), t))
        self.last_times_ms = (t[0], t[1])
        return out

    def set_prefill(self, rows: int) -> None:
        """0: the prompt token by token through the decode step (the reference's
        way, the parity mode); 16..64: in chunks of that many rows on the tf32
        tensor-core matmul (tq_qwen_set_prefill)."""
        _lib.check(_lib.load().tq_qwen_set_prefill(self.handle, rows))

    def set_sampling(self, temp: float, draws=None) -> None:
        """As Gpt2.set_sampling (tq_qwen_set_sampling; one GPU only)."""
        d = np.ascontiguousarray(draws if draws is not None else [], np.float64)
        _lib.check(_lib.load().tq_qwen_set_sampling(self.handle, float(temp), d.ctypes.data_as(ctypes.c_void_p) if len(d)
                                                    else None, len(d)))

    @property
    def exchange(self) -> str:
        """"none" (one GPU), "nccl" or "peer": how the decode step's partial
        sums meet (tq_qwen_exchange)."""
        k = ctypes.c_int()
        _lib.check(_lib.load().tq_qwen_exchange(self.handle, ctypes.byref(k)))
        return {_lib.TQ_EXCHANGE_NONE: "none", _lib.TQ_EXCHANGE_NCCL: "nccl", _lib.TQ_EXCHANGE_PEER: "peer"}[k.value]

    def free(self) -> None:
        if self.handle:
            _lib.load().tq_qwen_free(self.handle)
            self.handle = 0

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.free()
