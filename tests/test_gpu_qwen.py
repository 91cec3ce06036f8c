"""GPU Qwen2 int4 decode (tensor parallel) against the CPU oracle, through the
C ABI. Bar: identical greedy token ids (the -q4 loop of _example/qwen,
restated in oracle/tq_model.c) on small models, on the Qwen2.5-7B-shaped
config against committed golden ids, and over 2/4/8 GPUs when present."""
import ctypes
import glob
import os

import numpy as np
import pytest

from conftest import free_port

from oracle import oracle as O
from tensai_b200 import _lib
from tensai_b200.decode import QWEN_7B, Qwen, synth_tokens

pytestmark = pytest.mark.gpu

TINY = dict(n_layer=2, n_head=4, n_kv=2, d=256, ffn=512, vocab=1000, ctx=64, eps=1e-6, theta=1e6)
TINY_TP = dict(n_layer=2, n_head=8, n_kv=2, d=512, ffn=1024, vocab=1008, ctx=96, eps=1e-6, theta=1e6)
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _ndev():
    import torch
    return torch.cuda.device_count()


@pytest.fixture(scope="module", autouse=True)
def device():
    import torch
    torch.cuda.init()
    _lib.check(_lib.load().tq_set_device(0))


def _diverge(got, want, margins):
    bad = np.nonzero(np.asarray(got) != np.asarray(want))[0]
    if len(bad) == 0:
        return None
    i = int(bad[0])
    return f"token {i}: gpu {got[i]} oracle {want[i]}, oracle top-1 margin {float(margins[i]):.3g}"


@pytest.mark.parametrize("seed", [1, 2])
def test_tiny_qwen_matches_oracle(seed):
    prompt = synth_tokens(20, TINY["vocab"], seed)
    want, margins = O.qwen_generate(TINY, seed, 0.02, prompt, 30)
    with Qwen(TINY, seed) as m:
        got = m.generate(prompt, 30)
        again = m.generate(prompt, 30)
    assert np.array_equal(got, want), _diverge(got, want, margins)
    assert np.array_equal(again, got)


def test_single_token_prompt():
    prompt = synth_tokens(1, TINY["vocab"], 4)
    want, margins = O.qwen_generate(TINY, 4, 0.02, prompt, 8)
    with Qwen(TINY, 4) as m:
        got = m.generate(prompt, 8)
    assert np.array_equal(got, want), _diverge(got, want, margins)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "qwen7b_decode_golden_*.npz"))))
def test_qwen7b_shape_matches_golden_tokens(path):
    z = np.load(path)
    n_prompt, n_gen = len(z["prompt"]), len(z["tokens"])
    cfg = dict(QWEN_7B, ctx=n_prompt + n_gen)
    prompt = synth_tokens(n_prompt, cfg["vocab"], int(z["seed"]))
    assert np.array_equal(prompt, z["prompt"])
    with Qwen(cfg, int(z["seed"]), float(z["sigma"])) as m:
        got = m.generate(prompt, n_gen)
    assert np.array_equal(got, z["tokens"]), _diverge(got, z["tokens"], z["margins"])


@pytest.mark.parametrize("rows,seed", [(16, 1), (64, 2)])
def test_batched_prefill_tiny_qwen(rows, seed):
    """The prompt in chunks of `rows` positions (tq_qwen_set_prefill): 40
    prompt tokens (with rows=16 two full chunks and a ragged one of 8, which
    runs on the matvec kernels), each layer's matvecs as tf32 matmuls. The
    generated ids are the oracle's token-by-token ids here (the parity mode
    is checked alongside), and switching back restores the parity mode."""
    prompt = synth_tokens(40, TINY["vocab"], seed)
    want, margins = O.qwen_generate(TINY, seed, 0.02, prompt, 20)
    with Qwen(TINY, seed) as m:
        m.set_prefill(rows)
        got = m.generate(prompt, 20)
        m.set_prefill(0)
        ref = m.generate(prompt, 20)
    assert np.array_equal(ref, want), _diverge(ref, want, margins)
    assert np.array_equal(got, want), _diverge(got, want, margins)


def test_batched_prefill_rejects_bad_rows():
    with Qwen(TINY, 1) as m:
        for rows in (8, 65, -1):
            with pytest.raises(_lib.TensaiError) as e:
                m.set_prefill(rows)
            assert e.value.code == _lib.TQ_ERR_ARG


def test_qwen7b_shape_batched_prefill_agreement():
    """The 7B shape with its 64-token prompt as one 64-row chunk: the tf32
    matmuls change the prompt's hidden states slightly, so agreement with the
    golden token-by-token ids is reported (printed) rather than required
    beyond the first generated id."""
    z = np.load(os.path.join(GOLDEN, "qwen7b_decode_golden_64_32.npz"))
    n_prompt, n_gen = len(z["prompt"]), len(z["tokens"])
    cfg = dict(QWEN_7B, ctx=n_prompt + n_gen)
    with Qwen(cfg, int(z["seed"]), float(z["sigma"])) as m:
        m.set_prefill(64)
        got = m.generate(z["prompt"], n_gen)
    same = np.asarray(got) == np.asarray(z["tokens"])
    lead = int(np.argmin(same)) if not same.all() else len(same)
    print(f"batched prefill, 7B shape: {int(same.sum())}/{n_gen} ids equal to the token-by-token golden, "
          f"first {lead} in a row")
    assert got[0] == z["tokens"][0], _diverge(got, z["tokens"], z["margins"])


def _tp_worker(rank, world, port, q, cfg, seed, prompt, n, env, idle_rank, done):
    import torch
    import torch.distributed as dist

    from tensai_b200.decode import broadcast_nccl_id
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), **env)
    torch.cuda.set_device(rank)
    _lib.check(_lib.load().tq_set_device(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        nid = broadcast_nccl_id(dist)
        with Qwen(cfg, seed, 0.02, rank, world, nid) as m:
            if rank == idle_rank:  # joins the model but never the generate call
                q.put((rank, (m.exchange, "idle")))
                done.wait(60)
            else:
                kind = m.exchange
                try:
                    ids = m.generate(prompt, n).tolist()
                except Exception as e:
                    ids = repr(e)
                finally:
                    done.set()
                q.put((rank, (kind, ids)))
    except Exception as e:  # reported to the parent
        q.put((rank, (None, repr(e))))
    finally:
        dist.destroy_process_group()


def run_tp(cfg, seed, prompt, n, world, env=None, idle_rank=-1):
    """{rank: (exchange, ids or an error's repr)} of a world-GPU generate."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    done = ctx.Event()
    port = free_port()
    procs = [ctx.Process(target=_tp_worker, args=(r, world, port, q, cfg, seed, prompt, n, env or {}, idle_rank,
                                                  done)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    return got


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tensor_parallel_tiny_qwen_matches_oracle(world):
    if _ndev() < world:
        pytest.skip(f"needs {world} GPUs")
    prompt = synth_tokens(24, TINY_TP["vocab"], 3)
    want, margins = O.qwen_generate(TINY_TP, 3, 0.02, prompt, 40)
    got = run_tp(TINY_TP, 3, prompt, 40, world)
    for r in range(world):
        kind, ids = got[r]
        assert isinstance(ids, list), ids
        assert kind == "peer"
        assert np.array_equal(ids, want), (r, _diverge(ids, want, margins))


def test_tensor_parallel_nccl_exchange_matches_oracle():
    """TENSAI_QWEN_EXCHANGE=nccl keeps NCCL's all-reduce in the step: same ids."""
    if _ndev() < 2:
        pytest.skip("needs 2 GPUs")
    prompt = synth_tokens(24, TINY_TP["vocab"], 3)
    want, margins = O.qwen_generate(TINY_TP, 3, 0.02, prompt, 40)
    got = run_tp(TINY_TP, 3, prompt, 40, 2, env={"TENSAI_QWEN_EXCHANGE": "nccl"})
    for r in range(2):
        kind, ids = got[r]
        assert isinstance(ids, list), ids
        assert kind == "nccl"
        assert np.array_equal(ids, want), (r, _diverge(ids, want, margins))


def test_tensor_parallel_peer_exchange_times_out():
    """A rank that never joins generate: the other's exchange waits give up
    after 2 s and generate fails with TQ_ERR_TIMEOUT (nothing hangs; the idle
    rank keeps its memory mapped until the other has returned)."""
    if _ndev() < 2:
        pytest.skip("needs 2 GPUs")
    prompt = synth_tokens(4, TINY_TP["vocab"], 3)
    got = run_tp(TINY_TP, 3, prompt, 3, 2, env={"NCCL_NVLS_ENABLE": "0"}, idle_rank=1)
    assert got[1] == ("peer", "idle")
    kind, err = got[0]
    assert kind == "peer"
    assert isinstance(err, str) and "timed out" in err, err


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tensor_parallel_qwen7b_shape_matches_golden_tokens(world):
    """The Qwen2.5-7B shape sharded over 2, 4 or 8 GPUs (at 8, attention
    repeats over GPU pairs: 4 KV heads) gives the oracle's greedy ids."""
    if _ndev() < world:
        pytest.skip(f"needs {world} GPUs")
    z = np.load(os.path.join(GOLDEN, "qwen7b_decode_golden_64_32.npz"))
    n_prompt, n_gen = len(z["prompt"]), len(z["tokens"])
    cfg = dict(QWEN_7B, ctx=n_prompt + n_gen)
    prompt = synth_tokens(n_prompt, cfg["vocab"], int(z["seed"]))
    assert np.array_equal(prompt, z["prompt"])
    got = run_tp(cfg, int(z["seed"]), prompt, n_gen, world)
    for r in range(world):
        kind, ids = got[r]
        assert isinstance(ids, list), ids
        assert kind == "peer"
        assert np.array_equal(ids, z["tokens"]), (r, _diverge(ids, z["tokens"], z["margins"]))


# ---- checkpoint loading (tq_qwen_create_empty / tq_qwen_load_tensor) -----------

def _checkpoint(cfg, seed, sigma, scale_proj=1.0, norm=1.0):
    """The random-init model's weights in a Hugging Face Qwen2 checkpoint's
    names and [out, in] layout (F32), from the generator streams the engine
    draws them from; norm weights `norm`, biases 0; scale_proj multiplies the
    matrices that follow a norm (q, k, v, gate, up, lm head)."""
    d, ffn, vocab = cfg["d"], cfg["ffn"], cfg["vocab"]
    kv = cfg["n_kv"] * (d // cfg["n_head"])
    f32 = np.float32
    t = {"model.embed_tokens.weight": O.synth((vocab, d), seed, 1, sigma),
         "lm_head.weight": np.ascontiguousarray(O.synth((d, vocab), seed, 2, sigma).T) * f32(scale_proj),
         "model.norm.weight": np.full(d, norm, f32)}
    for l in range(cfg["n_layer"]):
        s0, p = 32 + 16 * l, f"model.layers.{l}."
        T = lambda shape, k: np.ascontiguousarray(O.synth(shape, seed, s0 + k, sigma).T)  # noqa: E731
        t[p + "self_attn.q_proj.weight"] = T((d, d), 0) * f32(scale_proj)
        t[p + "self_attn.k_proj.weight"] = T((d, kv), 1) * f32(scale_proj)
        t[p + "self_attn.v_proj.weight"] = T((d, kv), 2) * f32(scale_proj)
        t[p + "self_attn.o_proj.weight"] = T((d, d), 3)
        t[p + "mlp.gate_proj.weight"] = T((d, ffn), 4) * f32(scale_proj)
        t[p + "mlp.up_proj.weight"] = T((d, ffn), 5) * f32(scale_proj)
        t[p + "mlp.down_proj.weight"] = T((ffn, d), 6)
        for b, n in (("q", d), ("k", kv), ("v", kv)):
            t[p + f"self_attn.{b}_proj.bias"] = np.zeros(n, f32)
        t[p + "input_layernorm.weight"] = np.full(d, norm, f32)
        t[p + "post_attention_layernorm.weight"] = np.full(d, norm, f32)
    return t


def test_checkpoint_of_the_random_weights_gives_the_same_ids(tmp_path):
    """Loading, as checkpoint tensors, exactly the weights the random-init
    engine draws yields the same model: the same greedy ids, token by token
    and with the batched prefill."""
    from tensai_b200 import safetensors as ST
    p = str(tmp_path / "tiny.safetensors")
    ST.SaveFile(p, _checkpoint(TINY, 4, 0.02))
    prompt = synth_tokens(20, TINY["vocab"], 4)
    with Qwen(TINY, 4, 0.02) as ref, Qwen.from_checkpoint(TINY, p) as got:
        assert np.array_equal(got.generate(prompt, 24), ref.generate(prompt, 24))
        ref.set_prefill(16)
        got.set_prefill(16)
        assert np.array_equal(got.generate(prompt, 24), ref.generate(prompt, 24))


def test_checkpoint_norm_weights_feed_their_matrices(tmp_path):
    """Norm weights of 2 (every input, post-attention and final norm) against
    the matrices after them doubled: powers of two pass exactly through the
    int4 scales and the activation digits, so both checkpoints are the same
    model bit for bit if each norm weight reaches its own matrices."""
    from tensai_b200 import safetensors as ST
    pa, pb = str(tmp_path / "a.safetensors"), str(tmp_path / "b.safetensors")
    ST.SaveFile(pa, _checkpoint(TINY, 5, 0.02, norm=2.0))
    ST.SaveFile(pb, _checkpoint(TINY, 5, 0.02, scale_proj=2.0))
    prompt = synth_tokens(16, TINY["vocab"], 5)
    with Qwen.from_checkpoint(TINY, pa) as a, Qwen.from_checkpoint(TINY, pb) as b:
        assert np.array_equal(a.generate(prompt, 24), b.generate(prompt, 24))


def test_checkpoint_loading_errors():
    import torch
    c = TINY["d"]
    with Qwen(TINY, 1, 0.02) as m:
        with pytest.raises(_lib.TensaiError, match="random-init"):
            m.load_tensor("model.norm.weight", torch.ones(c, device="cuda"))
    m = Qwen.__new__(Qwen)
    h = ctypes.c_uint64()
    from tensai_b200.decode import QwenConfig
    _lib.check(_lib.load().tq_qwen_create_empty(ctypes.byref(QwenConfig(**TINY)), ctypes.byref(h)))
    m.handle, m.cfg, m.last_times_ms = h.value, dict(TINY), (0.0, 0.0)
    try:
        with pytest.raises(_lib.TensaiError, match="unknown Qwen2 tensor"):
            m.load_tensor("model.layers.0.self_attn.rotary.weight", torch.ones(c, device="cuda"))
        with pytest.raises(_lib.TensaiError, match="unknown Qwen2 tensor"):
            m.load_tensor("model.layers.9.input_layernorm.weight", torch.ones(c, device="cuda"))
        with pytest.raises(_lib.TensaiError, match="expected"):
            m.load_tensor("model.norm.weight", torch.ones(c + 1, device="cuda"))
        m.load_tensor("model.norm.weight", torch.ones(c, device="cuda", dtype=torch.bfloat16))
    finally:
        m.free()
