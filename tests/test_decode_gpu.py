"""KV-cache inference on the GPU (chessdecoder_b200.decode.BatchedBackbone,
csrc/decode.cu) against the reference's exported module (golden fixture) and
against the oracle at the full model size.

Tolerance: the caches, the GEMM inputs and the attention output are bf16 (the
reference runs fp16), so hidden states agree to a relative Frobenius error of
2e-2 (2 layers) / 3e-2 (12 layers) and a per-row cosine of 0.999 / 0.998."""
import numpy as np
import pytest
import torch

from chessdecoder_b200 import decode as D
from chessdecoder_b200 import kernels as K
from chessdecoder_b200.engine import ModelConfig, init_reference_weights
from oracle import decode as OD

from test_decode_cpu import G, golden_weights

pytestmark = pytest.mark.gpu


def _check(h, ref, rel_tol, cos_tol, what):
    h = h.detach().float().cpu().reshape(-1, h.shape[-1])
    ref = torch.as_tensor(ref).float().reshape(-1, h.shape[-1])
    rel = ((h - ref).norm() / ref.norm()).item()
    cos = torch.nn.functional.cosine_similarity(h, ref, dim=1).min().item()
    assert rel < rel_tol and cos > cos_tol, (what, rel, cos)


def _sd(cfg, named, seed=0):
    sd = init_reference_weights(cfg, seed)
    for k, v in named.items():
        sd[k] = torch.as_tensor(np.asarray(v, np.float32)).reshape(sd[k].shape)
    return sd


def test_decode_matches_reference_golden():
    w, gc = golden_weights()
    cfg = ModelConfig(vocab_size=gc["vocab_size"], embed_dim=gc["embed_dim"], num_heads=gc["num_heads"],
                      num_layers=gc["num_layers"], max_seq_len=gc["max_seq_len"], d_ff=gc["d_ff"],
                      num_fourier_freq=gc["num_fourier_freq"])
    bb = D.BatchedBackbone(cfg, batch_size=G["batch"], max_seq_len=gc["max_seq_len"], state_dict=_sd(cfg, w))
    K.get_error()
    for call in G["calls"]:
        h = getattr(bb, call["method"])(**call["inputs"])
        _check(h, call["hidden"], 2e-2, 0.999, call["method"])
    assert bb.causal_len == 8 + 3 and bb.prefix_len == 10 + 4 + 1
    assert K.get_error() == 0


def _full_scenario(rng, B, V):
    ids = lambda S: torch.from_numpy(rng.integers(0, V, (B, S)))  # noqa: E731
    calls = []
    S0 = 20
    num_real = torch.tensor([20, 17, 20, 12])
    om = torch.zeros(B, S0, dtype=torch.bool)
    om[1, 4] = om[3, 9] = True
    ov = torch.zeros(B, S0)
    ov[1, 4], ov[3, 9] = 0.6, -0.3
    calls.append(("causal_forward", dict(ids=ids(S0), pos=torch.arange(S0).repeat(B, 1), ov=ov, om=om,
                                         active=torch.ones(B, dtype=torch.bool), num_real=num_real)))
    pos = num_real.clone()
    for k in range(12):
        act = torch.from_numpy(rng.random(B) > 0.25)
        om1 = torch.zeros(B, 1, dtype=torch.bool)
        ov1 = torch.zeros(B, 1)
        if k % 4 == 1:
            om1[k % B, 0], ov1[k % B, 0] = True, float(rng.uniform(-1, 1))
        calls.append(("causal_incremental", dict(ids=ids(1), pos=pos[:, None].clone(), ov=ov1, om=om1, active=act)))
        pos = pos + act.long()
    calls.append(("causal_probe", dict(ids=ids(3), pos=torch.stack([pos, pos + 1, pos + 2], 1), ov=torch.zeros(B, 3),
                                       om=torch.zeros(B, 3, dtype=torch.bool))))
    S1 = 24
    blk = torch.from_numpy(np.repeat(np.arange(6), 4))
    m = torch.where(blk[None, :] <= blk[:, None], 0.0, -1e9).expand(B, 1, S1, S1).clone()
    calls.append(("prefix_forward", dict(ids=ids(S1), pos=torch.arange(S1).repeat(B, 1), mask=m, ov=torch.zeros(B, S1),
                                         om=torch.zeros(B, S1, dtype=torch.bool),
                                         active=torch.tensor([True, True, False, True]))))
    calls.append(("prefix_block_forward", dict(ids=ids(5), pos=torch.arange(S1, S1 + 5).repeat(B, 1),
                                               ov=torch.zeros(B, 5), om=torch.zeros(B, 5, dtype=torch.bool),
                                               active=torch.tensor([True, False, True, True]))))
    for k in range(3):
        calls.append(("prefix_incremental", dict(ids=ids(1), pos=torch.full((B, 1), S1 + 5 + k), ov=torch.zeros(B, 1),
                                                 om=torch.zeros(B, 1, dtype=torch.bool),
                                                 active=torch.tensor([True, True, k != 1, True]))))
    calls.append(("prefix_probe", dict(ids=ids(2), pos=torch.full((B, 2), S1 + 8), ov=torch.zeros(B, 2),
                                       om=torch.zeros(B, 2, dtype=torch.bool))))
    return calls


def test_decode_full_size_matches_oracle():
    """E=1024, 16 heads, 12 layers; q / k weights scaled by 4 so that the
    attention is far from uniform and the masks matter."""
    cfg = ModelConfig()
    B, max_len = 4, 96
    sd = init_reference_weights(cfg, 5)
    for i in range(cfg.num_layers):
        for n in ("q_proj", "k_proj"):
            sd[f"layers.{i}.attn.{n}.weight"] = sd[f"layers.{i}.attn.{n}.weight"] * 4.0
    bb = D.BatchedBackbone(cfg, batch_size=B, max_seq_len=max_len, state_dict=sd)
    w = {k: v.float().numpy() for k, v in sd.items()}
    ob = OD.Batched(w, dict(num_layers=cfg.num_layers, num_heads=cfg.num_heads, embed_dim=cfg.embed_dim,
                            max_seq_len=cfg.max_seq_len), B, max_len)
    K.get_error()
    for name, kw in _full_scenario(np.random.default_rng(2), B, cfg.vocab_size):
        h = getattr(bb, name)(**kw)
        ref = getattr(ob, name)(**{k: v.numpy() for k, v in kw.items()})
        _check(h, ref, 3e-2, 0.998, name)
    assert (bb.causal_len, bb.prefix_len) == (ob.causal_len, ob.prefix_len)
    assert K.get_error() == 0


def test_premarked_keys_and_cache_limit():
    """markCausalValidRange ahead of an incremental step keeps a pre-marked key
    valid for an inactive sequence (the reference's masked_fill only sets
    zeros); a step past the cache capacity is rejected on the host."""
    cfg = ModelConfig(num_layers=2)
    B, max_len = 2, 8
    sd = init_reference_weights(cfg, 1)
    bb = D.BatchedBackbone(cfg, batch_size=B, max_seq_len=max_len, state_dict=sd)
    w = {k: v.float().numpy() for k, v in sd.items()}
    ob = OD.Batched(w, dict(num_layers=2, num_heads=cfg.num_heads, embed_dim=cfg.embed_dim,
                            max_seq_len=cfg.max_seq_len), B, max_len)
    rng = np.random.default_rng(0)
    S0 = 6
    kw = dict(ids=torch.from_numpy(rng.integers(0, cfg.vocab_size, (B, S0))), pos=torch.arange(S0).repeat(B, 1),
              ov=torch.zeros(B, S0), om=torch.zeros(B, S0, dtype=torch.bool), active=torch.ones(B, dtype=torch.bool),
              num_real=torch.tensor([6, 6]))
    _check(bb.causal_forward(**kw), ob.causal_forward(**{k: v.numpy() for k, v in kw.items()}), 3e-2, 0.998, "fwd")
    both = torch.ones(B, dtype=torch.bool)
    bb.mark_causal_valid_range(S0, 1, both)
    ob.cbuf[both.numpy(), S0] = 0.0
    kw = dict(ids=torch.from_numpy(rng.integers(0, cfg.vocab_size, (B, 1))), pos=torch.full((B, 1), S0),
              ov=torch.zeros(B, 1), om=torch.zeros(B, 1, dtype=torch.bool), active=torch.tensor([True, False]))
    _check(bb.causal_incremental(**kw), ob.causal_incremental(**{k: v.numpy() for k, v in kw.items()}), 3e-2, 0.998,
           "incremental after pre-mark")
    kw["ids"] = torch.zeros(B, 2, dtype=torch.long)
    with pytest.raises(ValueError):
        bb.causal_probe(ids=kw["ids"], pos=torch.zeros(B, 2, dtype=torch.long), ov=None, om=None)
    assert K.get_error() == 0


def test_prefill_rows_above_split_threshold():
    """A prefill of more than 512 rows (the fused-epilogue GEMM path) followed
    by incremental steps (the split-K path), against the oracle."""
    cfg = ModelConfig(num_layers=4)
    B, max_len, S0 = 12, 64, 48
    sd = init_reference_weights(cfg, 9)
    for i in range(cfg.num_layers):
        for n in ("q_proj", "k_proj"):
            sd[f"layers.{i}.attn.{n}.weight"] = sd[f"layers.{i}.attn.{n}.weight"] * 4.0
    bb = D.BatchedBackbone(cfg, batch_size=B, max_seq_len=max_len, state_dict=sd)
    w = {k: v.float().numpy() for k, v in sd.items()}
    ob = OD.Batched(w, dict(num_layers=cfg.num_layers, num_heads=cfg.num_heads, embed_dim=cfg.embed_dim,
                            max_seq_len=cfg.max_seq_len), B, max_len)
    rng = np.random.default_rng(4)
    kw = dict(ids=torch.from_numpy(rng.integers(0, cfg.vocab_size, (B, S0))), pos=torch.arange(S0).repeat(B, 1),
              ov=torch.zeros(B, S0), om=torch.zeros(B, S0, dtype=torch.bool), active=torch.ones(B, dtype=torch.bool),
              num_real=torch.tensor([48, 40, 48, 33, 47, 48, 48, 21, 48, 48, 44, 48]))
    K.get_error()
    _check(bb.causal_forward(**kw), ob.causal_forward(**{k: v.numpy() for k, v in kw.items()}), 3e-2, 0.998,
           "prefill")
    pos = kw["num_real"].clone()
    for step in range(3):
        kw = dict(ids=torch.from_numpy(rng.integers(0, cfg.vocab_size, (B, 1))), pos=pos[:, None].clone(),
                  ov=torch.zeros(B, 1), om=torch.zeros(B, 1, dtype=torch.bool), active=torch.ones(B, dtype=torch.bool))
        _check(bb.causal_incremental(**kw), ob.causal_incremental(**{k: v.numpy() for k, v in kw.items()}), 3e-2,
               0.998, f"step {step}")
        pos += 1
    assert K.get_error() == 0


@pytest.mark.parametrize("use_graphs", [True, False])
def test_greedy_generation_matches_oracle(use_graphs):
    """Device-side greedy generation through the board head (causalBoardStep),
    replayed from a CUDA graph or run eagerly: each generated token, fed back
    teacher-forced into the oracle, is the oracle's argmax unless the oracle's
    top-2 margin is a near-tie."""
    from chessdecoder_b200 import vocab as V
    cfg = ModelConfig(num_layers=4)
    B, max_len, S0, n = 3, 48, 10, 12
    sd = init_reference_weights(cfg, 13)
    sd["board_head.weight"] = sd["board_head.weight"] * 30.0
    for i in range(cfg.num_layers):
        for nm in ("q_proj", "k_proj"):
            sd[f"layers.{i}.attn.{nm}.weight"] = sd[f"layers.{i}.attn.{nm}.weight"] * 4.0
    bb = D.BatchedBackbone(cfg, batch_size=B, max_seq_len=max_len, state_dict=sd, use_graphs=use_graphs)
    w = {k: v.float().numpy() for k, v in sd.items()}
    ob = OD.Batched(w, dict(num_layers=cfg.num_layers, num_heads=cfg.num_heads, embed_dim=cfg.embed_dim,
                            max_seq_len=cfg.max_seq_len), B, max_len)
    rng = np.random.default_rng(8)
    kw = dict(ids=torch.from_numpy(rng.integers(0, cfg.vocab_size, (B, S0))), pos=torch.arange(S0).repeat(B, 1),
              ov=torch.zeros(B, S0), om=torch.zeros(B, S0, dtype=torch.bool), active=torch.ones(B, dtype=torch.bool),
              num_real=torch.full((B,), S0))
    bb.causal_forward(**kw)
    ob.causal_forward(**{k: v.numpy() for k, v in kw.items()})
    lut = V.board_idx_to_full_idx
    first = torch.full((B, 1), V.token_to_idx["start_pos"] if "start_pos" in V.token_to_idx else 0)
    K.get_error()
    gen = bb.generate(first, torch.full((B, 1), S0), n, head="board_head", lut=lut).cpu()
    assert gen.shape == (n, B) and bb.causal_len == S0 + n
    assert K.get_error() == 0
    inv = {t: i for i, t in enumerate(lut)}
    ids = first.numpy()
    near_ties = 0
    for k in range(n):
        h = ob.causal_incremental(ids, np.full((B, 1), S0 + k), np.zeros((B, 1), np.float32),
                                  np.zeros((B, 1), bool), np.ones(B, bool))
        logits = h[:, 0] @ w["board_head.weight"].T + w["board_head.bias"]
        for b in range(B):
            got = inv[int(gen[k, b])]
            best = int(np.argmax(logits[b]))
            if got != best:
                margin = logits[b, best] - logits[b, got]
                assert margin < 0.02 * logits[b].std(), (k, b, got, best, margin)
                near_ties += 1
        ids = gen[k].numpy().reshape(B, 1)
    assert near_ties <= 2


@pytest.mark.parametrize("B,S0", [(2, 40), (12, 48), (3, 256)])
def test_unpadded_prefill_uses_training_attention(B, S0):
    """A causal prefill without padding into an empty cache (the training
    attention path), then incremental steps over the cache it wrote."""
    cfg = ModelConfig(num_layers=3)
    max_len = S0 + 4
    sd = init_reference_weights(cfg, 21)
    for i in range(cfg.num_layers):
        for nm in ("q_proj", "k_proj"):
            sd[f"layers.{i}.attn.{nm}.weight"] = sd[f"layers.{i}.attn.{nm}.weight"] * 4.0
    bb = D.BatchedBackbone(cfg, batch_size=B, max_seq_len=max_len, state_dict=sd)
    w = {k: v.float().numpy() for k, v in sd.items()}
    ob = OD.Batched(w, dict(num_layers=cfg.num_layers, num_heads=cfg.num_heads, embed_dim=cfg.embed_dim,
                            max_seq_len=cfg.max_seq_len), B, max_len)
    rng = np.random.default_rng(B * 100 + S0)
    om = torch.zeros(B, S0, dtype=torch.bool)
    om[0, 5] = True
    ov = torch.zeros(B, S0)
    ov[0, 5] = 0.4
    kw = dict(ids=torch.from_numpy(rng.integers(0, cfg.vocab_size, (B, S0))), pos=torch.arange(S0).repeat(B, 1),
              ov=ov, om=om, active=torch.ones(B, dtype=torch.bool), num_real=torch.full((B,), S0))
    K.get_error()
    _check(bb.causal_forward(**kw), ob.causal_forward(**{k: v.numpy() for k, v in kw.items()}), 3e-2, 0.998,
           "prefill")
    for step in range(2):
        kw = dict(ids=torch.from_numpy(rng.integers(0, cfg.vocab_size, (B, 1))), pos=torch.full((B, 1), S0 + step),
                  ov=torch.zeros(B, 1), om=torch.zeros(B, 1, dtype=torch.bool), active=torch.ones(B, dtype=torch.bool))
        _check(bb.causal_incremental(**kw), ob.causal_incremental(**{k: v.numpy() for k, v in kw.items()}), 3e-2,
               0.998, f"step {step}")
    assert K.get_error() == 0


def test_head_select_sampling_and_log_probs():
    """cdk_head_select: greedy = argmax; at a temperature the sample frequencies
    over 8192 identical rows follow softmax(logits / T) (each within 0.03, about
    4 standard deviations); the recorded log-probability is the unscaled
    log-softmax at the chosen index; the same seed repeats, another seed
    differs."""
    g = torch.Generator(device="cuda").manual_seed(3)
    V, R = 12, 8192
    base = torch.randn(V, device="cuda", generator=g) * 1.5
    logits = base.repeat(R, 1).contiguous()
    ids = torch.empty(R, dtype=torch.int64, device="cuda")
    lp = torch.empty(R, device="cuda")
    K.get_error()
    K.head_select(logits, ids, temperature=0.0, lp=lp)
    assert bool((ids == int(base.argmax())).all())
    ref_lp = torch.log_softmax(base, 0)
    assert torch.allclose(lp, ref_lp[ids], atol=1e-5)
    for T in (1.0, 0.6):
        seed = torch.tensor([12345], dtype=torch.int64, device="cuda")
        K.head_select(logits, ids, temperature=T, seed=seed, lp=lp)
        freq = torch.bincount(ids, minlength=V).float() / R
        assert (freq - torch.softmax(base / T, 0)).abs().max().item() < 0.03, T
        assert torch.allclose(lp, ref_lp[ids], atol=1e-5)
        again = torch.empty_like(ids)
        K.head_select(logits, again, temperature=T, seed=seed)
        assert torch.equal(again, ids)
        K.head_select(logits, again, temperature=T, seed=seed + 1)
        assert not torch.equal(again, ids)
    assert K.get_error() == 0


def test_head_select_never_samples_masked_columns():
    """Columns masked to -1e9 (illegal moves) are never sampled: about 1e9
    masked (row, column) draws across 64 seeds, where a uniform that rounded
    to 1 (a Gumbel term of +inf, probability 2^-24 per draw) would pick one."""
    R, V, legal = 8192, 1924, 12
    g = torch.Generator(device="cuda").manual_seed(9)
    logits = torch.full((R, V), -1e9, device="cuda")
    cols = torch.randperm(V, generator=g, device="cuda")[:legal]
    logits[:, cols] = torch.randn(R, legal, device="cuda", generator=g)
    ok = torch.zeros(V, dtype=torch.bool, device="cuda")
    ok[cols] = True
    ids = torch.empty(R, dtype=torch.int64, device="cuda")
    for s in range(64):
        K.head_select(logits, ids, temperature=1.0, seed=torch.tensor([1000 + s], dtype=torch.int64, device="cuda"))
        assert bool(ok[ids].all()), s
    assert K.get_error() == 0


def test_generate_with_temperature():
    """Sampled generation on the device: ids in the board vocabulary, and the
    recorded log-probabilities equal the oracle's log-softmax of the board head
    at the sampled tokens (teacher-forced).  (Runs are not bit-reproducible:
    the split-K projections reduce fp32 partial sums in no fixed order, so a
    near-tie of the sampling rule can go either way; the kernel-level test
    checks the seed.)"""
    from chessdecoder_b200 import vocab as V
    cfg = ModelConfig(num_layers=2)
    B, max_len, S0, n = 3, 64, 8, 10
    sd = init_reference_weights(cfg, 17)
    sd["board_head.weight"] = sd["board_head.weight"] * 10.0
    w = {k: v.float().numpy() for k, v in sd.items()}
    lut = V.board_idx_to_full_idx
    inv = {t: i for i, t in enumerate(lut)}
    rng = np.random.default_rng(5)
    prompt = torch.from_numpy(rng.integers(0, cfg.vocab_size, (B, S0)))
    bb = D.BatchedBackbone(cfg, batch_size=B, max_seq_len=max_len, state_dict=sd)
    kw = dict(ids=prompt, pos=torch.arange(S0).repeat(B, 1), ov=torch.zeros(B, S0),
              om=torch.zeros(B, S0, dtype=torch.bool), active=torch.ones(B, dtype=torch.bool),
              num_real=torch.full((B,), S0))
    bb.causal_forward(**kw)
    first = torch.full((B, 1), V.token_to_idx["start_pos"])
    K.get_error()
    ids, lps = bb.generate(first, torch.full((B, 1), S0), n, head="board_head", lut=lut, temperature=1.0, seed=99,
                           return_log_probs=True)
    ids, lps = ids.cpu(), lps.cpu()
    assert all(int(t) in inv for t in ids.flatten())
    ob = OD.Batched(w, dict(num_layers=cfg.num_layers, num_heads=cfg.num_heads, embed_dim=cfg.embed_dim,
                            max_seq_len=cfg.max_seq_len), B, max_len)
    ob.causal_forward(**{k: v.numpy() for k, v in kw.items()})
    cur = first.numpy()
    for k in range(n):
        h = ob.causal_incremental(cur, np.full((B, 1), S0 + k), np.zeros((B, 1), np.float32), np.zeros((B, 1), bool),
                                  np.ones(B, bool))
        logits = torch.from_numpy(h[:, 0] @ w["board_head.weight"].T + w["board_head.bias"])
        ref = torch.log_softmax(logits, 1)
        for b in range(B):
            assert abs(float(lps[k, b]) - float(ref[b, inv[int(ids[k, b])]])) < 0.05 + 0.02 * abs(float(lps[k, b]))
        cur = ids[k].numpy().reshape(B, 1)
    assert K.get_error() == 0


def test_value_heads_match_oracle():
    """WL / D value heads on the last hidden state (evalWlHead / evalDHead):
    bucket logits against Linear -> Mish -> Linear on the oracle's hidden state,
    the greedy bucket (unless a near-tie), its log-probability and centre value."""
    from chessdecoder_b200.engine import make_d_buckets, make_wl_buckets
    cfg = ModelConfig(num_layers=2)
    B, S0 = 4, 12
    sd = init_reference_weights(cfg, 23)
    for name in ("wl_head", "d_head"):
        sd[f"{name}.mlp.2.weight"] = sd[f"{name}.mlp.2.weight"] * 8.0
    bb = D.BatchedBackbone(cfg, batch_size=B, max_seq_len=32, state_dict=sd)
    w = {k: v.float().numpy() for k, v in sd.items()}
    ob = OD.Batched(w, dict(num_layers=cfg.num_layers, num_heads=cfg.num_heads, embed_dim=cfg.embed_dim,
                            max_seq_len=cfg.max_seq_len), B, 32)
    rng = np.random.default_rng(6)
    kw = dict(ids=torch.from_numpy(rng.integers(0, cfg.vocab_size, (B, S0))), pos=torch.arange(S0).repeat(B, 1),
              ov=torch.zeros(B, S0), om=torch.zeros(B, S0, dtype=torch.bool), active=torch.ones(B, dtype=torch.bool),
              num_real=torch.full((B,), S0))
    bb.causal_forward(**kw)
    h = ob.causal_forward(**{k: v.numpy() for k, v in kw.items()})[:, -1]
    K.get_error()
    for name, centers in (("wl_head", make_wl_buckets(cfg.n_buckets, cfg.wl_sigma)), ("d_head", make_d_buckets())):
        idx, val, lp, logits = bb.value_head(name)
        z = torch.from_numpy(h @ w[f"{name}.mlp.0.weight"].T + w[f"{name}.mlp.0.bias"])
        a = z * torch.tanh(torch.nn.functional.softplus(z))
        ref = a @ torch.from_numpy(w[f"{name}.mlp.2.weight"]).T + torch.from_numpy(w[f"{name}.mlp.2.bias"])
        _check(logits, ref, 3e-2, 0.998, name)
        ref_lp = torch.log_softmax(ref, 1)
        idx, val, lp = idx.cpu(), val.cpu(), lp.cpu()
        for b in range(B):
            best = int(ref[b].argmax())
            if int(idx[b]) != best:
                assert ref[b, best] - ref[b, int(idx[b])] < 0.02 * ref[b].std(), (name, b)
            assert abs(float(lp[b]) - float(ref_lp[b, int(idx[b])])) < 0.05 + 0.02 * abs(float(lp[b]))
            assert float(val[b]) == float(centers[int(idx[b])])
    assert K.get_error() == 0
