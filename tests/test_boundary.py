"""Drop-in boundary checks that need no GPU: the C ABI loads and exports every
declared symbol, host-side validation rejects bad arguments before any launch,
and the module tree / state-dict keys are the reference's."""

import ctypes
import os
import re

import pytest
import torch

import local_research_small_language_model_b200 as sd
from local_research_small_language_model_b200 import _lib
from local_research_small_language_model_b200.model import SparDAB200Model
from oracle.synthetic import SmallModelConfig, state_shapes

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    txt = open(os.path.join(REPO, "include", "spardab200.h")).read()
    return sorted(set(re.findall(r"SD_API\s+(?:const\s+char\s*\*|int)\s*(sd_\w+)\s*\(", txt)))


def test_library_exports_every_declared_symbol():
    lib = sd.load_library()
    decl = declared_symbols()
    assert len(decl) >= 12
    for name in decl:
        assert hasattr(lib, name), name
    assert sorted(_lib.exported_symbols()) == decl
    assert lib.sd_version() >= 1


def test_strerror_texts():
    lib = sd.load_library()
    for code in (0, -1, -2, -3, -4):
        assert lib.sd_strerror(code)
    assert lib.sd_strerror(-99) == b"unknown error"


def test_host_validation_rejects_bad_arguments():
    """Null pointers and bad shapes are refused before any CUDA call."""
    lib = sd.load_library()
    assert lib.sd_compress_blocks(None, 1, 1, 64, 4, 64, 0, 0, 0, 64, None, None) == -1
    assert lib.sd_topk_rows(None, 1, 8, 8, 4, None, None, None) == -1
    assert lib.sd_decode_attention(None, 1, 1, 12, 4, 64, 0, 0, None, None, 0, 0, 0, 64, None, None, 10, 1, 64,
                                   0.125, None, 0, 0, None, None) == -1
    # unsupported head_dim with otherwise valid-looking (non-null) pointers
    p = ctypes.c_void_p(16)
    assert lib.sd_decode_attention(p, 1, 1, 12, 4, 32, 0, 0, p, p, 0, 0, 0, 64, p, p, 10, 1, 64, 0.125, p, 0, 0,
                                   None, None) == -2
    assert lib.sd_decode_select(None, 0, 0, 0, None, 0, 0, 0, 1, 4, 64, 100, 64, 8, 7, p, p, 10, None) == -1


def test_ops_refuse_cpu_tensors():
    k = torch.zeros(1, 64, 4, 64)
    with pytest.raises(ValueError, match="CUDA"):
        sd.ops.compress_blocks(k, 64)
    with pytest.raises(ValueError, match="CUDA"):
        sd.KVBlockCompressor(64, 64, 64)(k)


def test_model_state_dict_matches_reference_layout():
    m = SparDAB200Model(sd.ModelConfig(block_size=64, top_k_blocks=8))
    assert sum(p.numel() for p in m.parameters()) == 102_451_968  # reference tests/test_model.py:9-28
    sc = SmallModelConfig(vocab_size=32000, n_layer=12)
    ref = state_shapes(sc)
    got = {k: tuple(v.shape) for k, v in m.state_dict().items()}
    assert got == ref


def test_install_swaps_attention_modules():
    cfg = sd.ModelConfig(n_layer=2, block_size=64, top_k_blocks=8)
    m = SparDAB200Model(cfg)
    w = m.layers[1].attention.wq.weight.clone()
    sd.install(m, rule="absolute")
    assert isinstance(m.layers[1].attention, sd.B200SparseAttention)
    assert m.layers[1].attention.rule == "absolute"
    assert torch.equal(m.layers[1].attention.wq.weight, w)


def test_install_into_reference_model():
    """The reference's own model accepts the backend (module swap; CPU only,
    so no forward).  SPARDA_REFERENCE names the reference checkout; skipped
    where it is unset or absent."""
    ref = os.environ.get("SPARDA_REFERENCE", "")
    if not ref or not os.path.isdir(os.path.join(ref, "model")):
        pytest.skip("reference checkout not present")
    import sys
    sys.path.insert(0, ref)
    from model.config import ModelConfig as RC
    from model.model import SparDAResearchModel
    r = SparDAResearchModel(RC(n_layer=2, block_size=64, top_k_blocks=8, attention_backend="sparse"))
    before = {k: v.clone() for k, v in r.state_dict().items()}
    sd.install(r)
    after = r.state_dict()
    assert set(before) == set(after)
    for k in before:
        assert torch.equal(before[k], after[k]), k


def test_selector_rule_validation():
    with pytest.raises(ValueError):
        sd.B200SparseAttention(sd.ModelConfig(), 1, rule="bogus")


def test_rope_tables_stay_fp32_under_module_cast():
    """model.to(bfloat16) must not turn the RoPE tables into 16-bit buffers: the
    fused decode kernel reads them as fp32 (a 16-bit table would be misread and
    read past its end).  The boundary check rejects such tables outright."""
    from local_research_small_language_model_b200 import ops
    rot = sd.RotaryEmbedding(64, 256).to(torch.bfloat16)
    assert rot.cos.dtype == torch.float32 and rot.sin.dtype == torch.float32
    ref_cos, _ = sd.rope.precompute_rope_freqs(64, 256)
    assert torch.equal(rot.cos, ref_cos)
    from local_research_small_language_model_b200.model import SparDAB200Model
    m = SparDAB200Model(sd.ModelConfig(n_layer=1, vocab_size=64)).to(torch.bfloat16)
    assert m.rotary_emb.cos.dtype == torch.float32
    with pytest.raises(TypeError):
        ops._rope_tables(rot.cos.to(torch.bfloat16), rot.sin.to(torch.bfloat16), 64, 128)
    with pytest.raises(ValueError):
        ops._rope_tables(rot.cos, rot.sin, 64, 1024)
    ops._rope_tables(rot.cos, rot.sin, 64, 256)


def test_prefill_wrappers_reject_mismatched_shapes_before_launch():
    """ops.prefill_attention / prefill_attention_backward check every shape the
    kernels index by before anything reaches the device (so a wrong list or
    gradient tensor cannot make a kernel read out of bounds); correctly shaped
    CPU tensors get as far as the CUDA check."""
    import pytest
    import torch
    from local_research_small_language_model_b200 import ops

    b, t, hq, hkv, d = 2, 130, 6, 2, 64
    q = torch.zeros(b, t, hq, d)
    k = torch.zeros(b, hkv, t, d)
    lists = torch.zeros(b, hkv, 3, 10, dtype=torch.int32)
    counts = torch.zeros(b, hkv, 3, dtype=torch.int32)
    topk = torch.zeros(b, hkv, t, 8, dtype=torch.int64)
    bad = {
        "k and v must be": dict(k=torch.zeros(b, hkv, t - 1, d)),
        "multiple of kv heads": dict(k=torch.zeros(b, 4, t, d)),
        "lists must be": dict(lists=torch.zeros(b, hkv, 2, 10, dtype=torch.int32)),
        "contiguous int32": dict(counts=torch.zeros(b, hkv, 3, dtype=torch.int64)),
        "topk must be": dict(topk=torch.zeros(b, hkv, t - 1, 8, dtype=torch.int64)),
    }
    for msg, over in bad.items():
        a = dict(q=q, k=k, v=k, lists=lists, counts=counts, topk=topk)
        a.update(over)
        if "k" in over:
            a["v"] = a["k"]
        with pytest.raises(ValueError, match=msg):
            ops.prefill_attention(a["q"], a["k"], a["v"], a["lists"], a["counts"], 64, a["topk"])
    with pytest.raises(ValueError, match="dout must have"):
        ops.prefill_attention_backward(q, k, k, torch.zeros(b, t, hq, d - 1), lists, counts, 64, topk)
    # a cache view holding more sequences and positions than the prompt is fine
    big = torch.zeros(b + 1, hkv, t + 64, d)[:, :, :t + 10]
    for call in (lambda: ops.prefill_attention(q, big, big, lists, counts, 64, topk),
                 lambda: ops.prefill_attention_backward(q, big, big, q, lists, counts, 64, topk)):
        with pytest.raises(ValueError, match="need CUDA tensors"):
            call()


def test_decode_and_append_wrappers_reject_mismatched_shapes():
    """ops.decode_attention and ops.kv_append check the shapes their kernels
    index by before the CUDA check (the stores and sums may be sized for more
    sequences than the call uses)."""
    import pytest
    import torch
    from local_research_small_language_model_b200 import ops

    q = torch.zeros(2, 12, 64)
    kc = torch.zeros(2, 4, 256, 64)
    sel, cnt = torch.zeros(2, 4, 10, dtype=torch.int32), torch.zeros(2, 4, dtype=torch.int32)
    with pytest.raises(ValueError, match="do not fit"):
        ops.decode_attention(q, kc[:1], kc[:1], sel, cnt, 100, 64)
    with pytest.raises(ValueError, match="do not fit"):
        ops.decode_attention(q, kc, kc, sel, cnt, 300, 64)
    with pytest.raises(ValueError, match="sel must be"):
        ops.decode_attention(q, kc, kc, sel[:, :3], cnt, 100, 64)
    with pytest.raises(ValueError, match="need CUDA tensors"):
        ops.decode_attention(q, kc, kc, sel, cnt, 100, 64)
    xk = torch.zeros(2, 70, 4, 64)
    store = torch.zeros(3, 4, 256, 64)
    sums = torch.zeros(3, 4, 4, 64)
    with pytest.raises(ValueError, match="do not fit"):
        ops.kv_append(xk, xk, store[:, :2].contiguous(), store[:, :2].contiguous(), sums, 0, 64)
    with pytest.raises(ValueError, match="do not fit"):
        ops.kv_append(xk, xk, store, store, sums.double(), 0, 64)
    with pytest.raises(ValueError, match="alike"):
        ops.kv_append(xk, xk[:, :69], store, store, sums, 0, 64)
    with pytest.raises(ValueError, match="need CUDA tensors"):
        ops.kv_append(xk, xk, store[:2], store[:2], sums, 0, 64)


def test_gather_and_select_wrappers_reject_mismatched_shapes():
    import pytest
    import torch
    from local_research_small_language_model_b200 import ops

    k = torch.zeros(2, 4, 640, 64)
    with pytest.raises(ValueError, match="indices"):
        ops.gather_kv_blocks(k, k, torch.zeros(1, 4, 10, dtype=torch.int64), 64)
    with pytest.raises(ValueError, match="pinned"):  # well-shaped host K/V: the pinned-host rule applies next
        ops.gather_kv_blocks(k, k, torch.zeros(2, 4, 10, dtype=torch.int64), 64)
    f = torch.zeros(2, 1, 4, 64)
    with pytest.raises(ValueError, match="reps be"):
        ops.decode_select(f, torch.zeros(2, 9, 4, 64), 600, 2, 4, 64, 64, 8)  # 600 tokens = 10 blocks
    with pytest.raises(ValueError, match="need CUDA tensors"):
        ops.decode_select(f, torch.zeros(2, 10, 4, 64), 600, 2, 4, 64, 64, 8)


def test_rope_transpose_is_rope_with_negated_sin():
    """The backward of RoPE that the training path uses (_RopeQK: the same
    rotation with -sin) equals autograd's gradient through the reference-order
    rotation (apply_rotary_emb, fp32, CPU)."""
    import torch
    from local_research_small_language_model_b200.rope import apply_rotary_emb, precompute_rope_freqs

    torch.manual_seed(0)
    cos, sin = precompute_rope_freqs(64, 200)
    q = torch.randn(2, 37, 12, 64, dtype=torch.float64, requires_grad=True)
    k = torch.randn(2, 37, 4, 64, dtype=torch.float64, requires_grad=True)
    gq, gk = torch.randn(2, 37, 12, 64, dtype=torch.float64), torch.randn(2, 37, 4, 64, dtype=torch.float64)
    c64, s64 = cos.double(), sin.double()
    for offset in (0, 100):
        qr, kr = apply_rotary_emb(q, k, c64, s64, offset)
        dq, dk = torch.autograd.grad((qr * gq).sum() + (kr * gk).sum(), (q, k))
        tq, tk = apply_rotary_emb(gq, gk, c64, -s64, offset)
        torch.testing.assert_close(tq, dq, rtol=0, atol=1e-12)
        torch.testing.assert_close(tk, dk, rtol=0, atol=1e-12)
