"""CPU tests of the host logic: weight init order, batch index lists, flat
parameter layout, and that libcdk.so loads and exports every declared symbol."""
import re
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[1]
SMALL = dict(embed_dim=256, num_heads=4, num_layers=2, max_seq_len=256, d_ff=384)


def test_init_matches_reference_construction_order():
    from chessdecoder_b200.engine import ModelConfig, init_reference_weights
    from oracle.model import OracleChessDecoder
    cfg = ModelConfig(**SMALL)
    sd = init_reference_weights(cfg, seed=0)
    torch.manual_seed(0)
    ref = OracleChessDecoder(cfg.vocab_size, **SMALL).state_dict()
    for k, v in ref.items():
        if k.endswith("bucket_centers"):
            continue
        assert k in sd, k
        assert torch.equal(sd[k], v), k
    assert set(sd) == {k for k in ref if not k.endswith("bucket_centers")}


def test_param_store_layout():
    from chessdecoder_b200.engine import ModelConfig, ParamStore, param_specs
    cfg = ModelConfig(**SMALL)
    st = ParamStore(cfg, "cpu")
    # q|k|v and w1|w3 packed back to back
    for i in range(cfg.num_layers):
        p = f"layers.{i}."
        oq, _, nq = st.offsets[p + "attn.q_proj.weight"]
        assert st.offsets[p + "attn.k_proj.weight"][0] == oq + nq
        assert st.offsets[p + "attn.v_proj.weight"][0] == oq + 2 * nq
        o1, _, n1 = st.offsets[p + "mlp.w1.weight"]
        assert st.offsets[p + "mlp.w3.weight"][0] == o1 + n1
    for name, (off, shape, n) in st.offsets.items():
        assert off % 64 == 0 or name.endswith(("k_proj.weight", "v_proj.weight", "w3.weight")), name
    # every parameter in the reference (but the thinking head) appears exactly once
    names = [n for n, _ in param_specs(cfg)]
    assert len(names) == len(set(names))
    total = sum(int(np.prod(s)) for _, s in param_specs(cfg))
    assert st.numel >= total


def test_full_size_param_count():
    from chessdecoder_b200.engine import ModelConfig, param_specs
    cfg = ModelConfig()
    n = sum(int(np.prod(s)) for _, s in param_specs(cfg))
    # 113,821,305 trainable parameters in the reference minus the 1924*1025 thinking head
    assert n + 1924 * 1024 + 1924 == 115_793_405 or n > 100_000_000


def test_host_index_lists_match_reference_semantics():
    from chessdecoder_b200 import data
    from chessdecoder_b200.engine import _host_index_lists
    batch = data.synthetic_batches(1, 4, 256, seed=5)[0]
    lists, B, S = _host_index_lists(batch)
    mm = batch["move_mask"]
    assert lists["prow"].size == int(mm.sum())
    assert (lists["prow"] >= B * S).all()
    # WL rows are stm+1 of move rows (clamped)
    bb, ss = np.nonzero(mm.numpy())
    assert np.array_equal(lists["wrow"] - B * S, bb * S + np.minimum(ss + 1, S - 1))
    # board weights: target valid and at/after first move
    bt = batch["board_target_ids"].numpy()
    w = lists["board_w"].reshape(B, S)
    assert ((w > 0) <= (bt != -100)).all()
    # norms
    assert np.isclose(lists["norms"][0], 1.0 / (mm.sum().item() + 1e-8))


def test_library_exports_every_declared_symbol():
    import ctypes
    from chessdecoder_b200 import _lib
    header = (ROOT / "include" / "cdk.h").read_text()
    declared = set(re.findall(r"\b(cdk_[a-z0-9_]+)\s*\(", header))
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in declared:
        assert hasattr(lib, name), name
    assert declared <= set(_lib.SIGNATURES), declared - set(_lib.SIGNATURES)
    assert _lib.load().cdk_version() >= 1


def test_ops_refuse_cpu_tensors():
    import pytest
    from chessdecoder_b200 import kernels
    x = torch.zeros(4, 1024)
    with pytest.raises(RuntimeError):
        kernels.rmsnorm_fwd(x, torch.ones(1024))


def test_ctypes_signatures_match_header_arity():
    """Every C-ABI declaration in include/cdk.h has as many parameters as the
    ctypes binding in chessdecoder_b200/_lib.py passes (a mismatch would shift
    every later argument silently)."""
    from chessdecoder_b200 import _lib
    header = (ROOT / "include" / "cdk.h").read_text()
    header = re.sub(r"/\*.*?\*/", "", header, flags=re.S)
    for m in re.finditer(r"\b(cdk_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", header):
        name, params = m.group(1), " ".join(m.group(2).split())
        n = 0 if params in ("", "void") else params.count(",") + 1
        assert name in _lib.SIGNATURES, name
        assert len(_lib.SIGNATURES[name][1]) == n, (name, n, len(_lib.SIGNATURES[name][1]))


def test_pipelined_steps_reads_every_step_in_order():
    """engine.pipelined_steps keeps one step in flight and yields every step's
    losses in order (host tensors on a CPU-only run)."""
    import torch
    from chessdecoder_b200.engine import pipelined_steps
    calls = []

    def fake_step(b, metrics):
        calls.append(b)
        return torch.full((5,), float(b))

    it = pipelined_steps(fake_step, iter(range(4)))
    i0, l0 = next(it)
    assert calls == [0, 1] and i0 == 0 and torch.equal(l0, torch.zeros(5))  # step 1 enqueued before step 0 is read
    rest = list(it)
    assert [i for i, _ in rest] == [1, 2, 3] and [float(l[0]) for _, l in rest] == [1.0, 2.0, 3.0]
    assert list(pipelined_steps(fake_step, iter([]))) == []
