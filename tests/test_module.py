"""The drop-in ``ChessDecoder`` module (chessdecoder_b200.model) against the
reference contract of chessdecoder/models/model.py:55-194 and the loop of
chessdecoder/train/train.py:157-253.

CPU tests: constructor, attribute tree, state-dict keys and initial weights
(same ``torch.manual_seed`` -> same tensors as the oracle's construction, which
restates the reference order), the ValueError of prefix mode without
block_id, and the refusal of CPU tensors.

GPU tests: the reference loop body, written as train.py writes it (autocast
fp16 + GradScaler, heads called as modules, soft_bucket_loss and
prepare_fourier_inputs from this package), against the fp32 oracle step:
losses within 1e-2 relative and gradient cosine >= 0.999 for every
parameter; a few torch.optim.AdamW steps against the fused TrainStep; the
forward's hidden states against the oracle's; the soft-bucket loss kernel;
average_gradients over a one-rank NCCL group.
"""
import socket

import pytest
import torch

SMALL = dict(embed_dim=256, num_heads=4, num_layers=2, max_seq_len=256, d_ff=384)
IGNORE_INDEX = -100


def _cosine(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return (a @ b / (a.norm() * b.norm()).clamp_min(1e-30)).item()


def _models(seed=0, cfg_kw=SMALL):
    from chessdecoder_b200 import vocab as V
    from chessdecoder_b200.model import ChessDecoder
    from oracle.model import OracleChessDecoder
    torch.manual_seed(seed)
    ours = ChessDecoder(V.vocab_size, **cfg_kw)
    torch.manual_seed(seed)
    ref = OracleChessDecoder(V.vocab_size, **cfg_kw)
    return ours, ref


def test_state_dict_and_init_match_reference_construction():
    ours, ref = _models()
    a, b = ours.state_dict(), ref.state_dict()
    assert set(a) == set(b)
    for k in a:
        assert a[k].shape == b[k].shape, k
        assert torch.equal(a[k], b[k]), k
    # the attribute paths read by the reference export code
    l0 = ours.layers[0]
    for m in (l0.attn.q_proj, l0.attn.k_proj, l0.attn.v_proj, l0.attn.output_proj, l0.mlp.w1, l0.mlp.w2,
              l0.mlp.w3, ours.board_head, ours.policy_head, ours.thinking_policy_head, ours.wl_head.mlp[0],
              ours.wl_head.mlp[2], ours.d_head.mlp[0], ours.fourier_encoder.proj):
        assert isinstance(m, torch.nn.Linear)
    assert l0.sa_norm.scale.shape == (SMALL["embed_dim"],)
    assert l0.attn.pos_embeddings is ours.layers[1].attn.pos_embeddings
    assert ours.wl_bucket_centers.shape == (100,) and ours.d_bucket_centers.shape == (100,)


def test_forward_errors_on_cpu():
    ours, _ = _models()
    x = torch.zeros(1, 8, dtype=torch.long)
    with pytest.raises(ValueError):
        ours(x, mask_type="prefix")
    with pytest.raises(RuntimeError):
        ours(x)
    with pytest.raises(RuntimeError):
        ours.board_head(torch.zeros(2, SMALL["embed_dim"]))


def test_discretize_and_prepare_fourier_inputs_match_oracle():
    from chessdecoder_b200.model import prepare_fourier_inputs
    from oracle.step import prepare_fourier_inputs as ref_prep
    ours, ref = _models()
    g = torch.Generator().manual_seed(1)
    wl_t = torch.rand(3, 40, generator=g) * 2 - 1
    d_t = torch.rand(3, 40, generator=g)
    wl_p = torch.rand(3, 40, generator=g) < 0.2
    d_p = torch.rand(3, 40, generator=g) < 0.2
    a = prepare_fourier_inputs(ours, wl_t, d_t, wl_p, d_p)
    b = ref_prep(ref, wl_t, d_t, wl_p, d_p)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


# ---------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------
def _train_py_losses(model, b, soft_bucket_loss, prepare_fourier_inputs, use_amp, weights=(5.0, 1.0, 1.0, 1.0)):
    """The loss block of train.py:167-241, verbatim in structure."""
    from chessdecoder_b200 import vocab as V
    move_w, board_w, wl_w, d_w = weights
    dev = b["input_ids"].device
    input_ids, board_target_ids, move_target_ids = b["input_ids"], b["board_target_ids"], b["move_target_ids"]
    move_mask, wl_positions, d_positions = b["move_mask"], b["wl_positions"], b["d_positions"]
    wl_targets, d_targets, wdl_valid, block_id = b["wl_targets"], b["d_targets"], b["wdl_valid"], b["block_id"]
    board_ce_fn = torch.nn.CrossEntropyLoss(ignore_index=IGNORE_INDEX, reduction="none")
    move_ce_fn = torch.nn.CrossEntropyLoss(ignore_index=IGNORE_INDEX, reduction="none")
    with torch.autocast(device_type="cuda", dtype=torch.float16, enabled=use_amp):
        wl_in, d_in = prepare_fourier_inputs(model, wl_targets, d_targets, wl_positions, d_positions)
        h_causal = model(input_ids, mask_type="causal", wl_values=wl_in, d_values=d_in,
                         wl_positions=wl_positions, d_positions=d_positions)
        board_logits = model.board_head(h_causal)
        board_mask = board_target_ids != IGNORE_INDEX
        first_move_idx = move_mask.int().argmax(dim=1)
        has_moves = move_mask.any(dim=1)
        first_move_idx[~has_moves] = move_mask.size(1)
        indices = torch.arange(move_mask.size(1), device=dev).unsqueeze(0)
        board_mask = board_mask & (~(indices < first_move_idx.unsqueeze(1)))
        ce_board = board_ce_fn(board_logits.view(-1, V.board_vocab_size), board_target_ids.view(-1))
        board_loss = (ce_board.view(board_target_ids.shape) * board_mask.float()).sum() / (board_mask.sum() + 1e-8)
        h_prefix = model(input_ids, mask_type="prefix", block_id=block_id, wl_values=wl_in, d_values=d_in,
                         wl_positions=wl_positions, d_positions=d_positions)
        move_logits = model.policy_head(h_prefix)
        ce_move = move_ce_fn(move_logits.view(-1, V.move_vocab_size), move_target_ids.view(-1))
        move_loss = (ce_move.view(move_target_ids.shape) * move_mask.float()).sum() / (move_mask.sum() + 1e-8)
        nz = move_mask.nonzero(as_tuple=False)
        if nz.shape[0] > 0:
            seq = (nz[:, 1] + 1).clamp(max=h_prefix.shape[1] - 1)
            wl_logits = model.wl_head(h_prefix[nz[:, 0], seq])
            wl_loss = soft_bucket_loss(wl_logits, wl_targets[move_mask], model.wl_bucket_centers,
                                       wdl_valid[move_mask])
        else:
            wl_loss = torch.tensor(0.0, device=dev)
        if wl_positions.any():
            d_logits = model.d_head(h_prefix[wl_positions])
            d_loss = soft_bucket_loss(d_logits, d_targets[d_positions], model.d_bucket_centers,
                                      wdl_valid[d_positions])
        else:
            d_loss = torch.tensor(0.0, device=dev)
        total = move_w * move_loss + board_w * board_loss + wl_w * wl_loss + d_w * d_loss
    return {"total": total, "move": move_loss, "board": board_loss, "wl": wl_loss, "d": d_loss}


def _batch(B, S, seed=3):
    from chessdecoder_b200 import data
    return data.synthetic_batches(1, B, S, seed=seed)[0]


@pytest.mark.gpu
@pytest.mark.parametrize("use_amp", [False, True])
def test_train_py_loop_matches_oracle(use_amp):
    from chessdecoder_b200.model import prepare_fourier_inputs, soft_bucket_loss
    from oracle.step import step_losses
    ours, ref = _models()
    ours.cuda()
    batch = _batch(4, SMALL["max_seq_len"])
    out_ref = step_losses(ref, batch)
    out_ref["total"].backward()
    b = {k: v.cuda() for k, v in batch.items()}
    opt = torch.optim.AdamW(ours.parameters(), lr=3e-4, weight_decay=0.1)
    scaler = torch.amp.GradScaler("cuda", enabled=use_amp)
    out = _train_py_losses(ours, b, soft_bucket_loss, prepare_fourier_inputs, use_amp)
    scaler.scale(out["total"]).backward()
    scaler.unscale_(opt)
    for n in ("move", "board", "wl", "d"):
        r = float(out_ref[n].detach())
        got = float(out[n].detach())
        assert abs(got - r) <= 1e-2 * max(abs(r), 1e-6), (n, got, r)
    rp = dict(ref.named_parameters())
    for name, p in ours.named_parameters():
        if name.startswith("thinking_policy_head"):
            assert p.grad is None
            continue
        assert p.grad is not None, name
        c = _cosine(p.grad.cpu(), rp[name].grad)
        assert c >= 0.999, (name, c)
    # the optimizer step goes through (grads finite, no inf skip)
    torch.nn.utils.clip_grad_norm_(ours.parameters(), max_norm=10.0)
    scaler.step(opt)
    scaler.update()
    opt.zero_grad(set_to_none=True)


@pytest.mark.gpu
def test_module_with_torch_adamw_tracks_fused_step():
    """Three steps of module + torch.optim.AdamW + clip against three fused
    TrainStep steps from the same weights on the same batches."""
    from chessdecoder_b200 import data
    from chessdecoder_b200.engine import ModelConfig, TrainStep
    from chessdecoder_b200.model import prepare_fourier_inputs, soft_bucket_loss
    ours, _ = _models()
    cfg = ModelConfig(**SMALL)
    fused = TrainStep(cfg, device="cuda", state_dict={k: v.clone() for k, v in ours.state_dict().items()})
    ours.cuda()
    opt = torch.optim.AdamW(ours.parameters(), lr=3e-4, weight_decay=0.1)
    batches = data.synthetic_batches(3, 4, SMALL["max_seq_len"], seed=11)
    for i, batch in enumerate(batches):
        b = {k: v.cuda() for k, v in batch.items()}
        out = _train_py_losses(ours, b, soft_bucket_loss, prepare_fourier_inputs, use_amp=False)
        out["total"].backward()
        torch.nn.utils.clip_grad_norm_(ours.parameters(), max_norm=10.0)
        opt.step()
        opt.zero_grad(set_to_none=True)
        lf = fused.step(batch).cpu()
        for j, n in enumerate(("move", "board", "wl", "d")):
            r = float(lf[j])
            got = float(out[n].detach())
            assert abs(got - r) <= 1e-2 * max(abs(r), 1e-6), (i, n, got, r)
    # the flat store saw the optimizer's in-place updates
    sd = fused.store.state_dict()
    for name, p in ours.named_parameters():
        if name.startswith("thinking_policy_head"):
            continue
        c = _cosine(p.detach().cpu(), sd[name].cpu())
        assert c >= 0.9999, (name, c)


@pytest.mark.gpu
@pytest.mark.parametrize("mask_type", ["causal", "prefix"])
def test_forward_hidden_states_match_oracle(mask_type):
    ours, ref = _models()
    ours.cuda()
    batch = _batch(3, 200, seed=5)
    kw = dict(mask_type=mask_type, wl_values=batch["wl_targets"], d_values=batch["d_targets"],
              wl_positions=batch["wl_positions"], d_positions=batch["d_positions"])
    if mask_type == "prefix":
        kw["block_id"] = batch["block_id"]
    with torch.no_grad():
        h_ref = ref(batch["input_ids"], **kw)
        h = ours(batch["input_ids"].cuda(), **{k: (v.cuda() if torch.is_tensor(v) else v) for k, v in kw.items()})
    assert h.shape == h_ref.shape and h.dtype == torch.float32
    err = (h.cpu() - h_ref).norm() / h_ref.norm()
    assert err < 2e-2, float(err)


@pytest.mark.gpu
def test_soft_bucket_loss_kernel_matches_oracle():
    from chessdecoder_b200.engine import make_wl_buckets
    from chessdecoder_b200.model import soft_bucket_loss
    from oracle.step import soft_bucket_loss as ref_loss
    g = torch.Generator().manual_seed(0)
    n = 300
    logits = torch.randn(n, 100, generator=g) * 3
    tgt = torch.rand(n, generator=g) * 2.2 - 1.1  # includes values outside the centre range
    valid = torch.rand(n, generator=g) < 0.8
    c = make_wl_buckets()
    lr_ = logits.clone().requires_grad_(True)
    r = ref_loss(lr_, tgt, c, valid)
    r.backward()
    lc = logits.cuda().requires_grad_(True)
    v = soft_bucket_loss(lc, tgt.cuda(), c.cuda(), valid.cuda())
    v.backward()
    vf, rf = float(v.detach()), float(r.detach())
    assert abs(vf - rf) <= 1e-5 * max(1.0, abs(rf))
    assert torch.allclose(lc.grad.cpu(), lr_.grad, atol=1e-6, rtol=1e-4)
    # no valid rows -> constant 0 without a graph
    z = soft_bucket_loss(lc, tgt.cuda(), c.cuda(), torch.zeros(n, dtype=torch.bool, device="cuda"))
    assert float(z) == 0.0 and not z.requires_grad


@pytest.mark.gpu
def test_average_gradients_one_rank_uses_flat_buffer():
    import torch.distributed as dist
    from chessdecoder_b200.distributed import average_gradients
    from chessdecoder_b200.model import prepare_fourier_inputs, soft_bucket_loss
    ours, _ = _models()
    ours.cuda()
    b = {k: v.cuda() for k, v in _batch(2, 256).items()}
    out = _train_py_losses(ours, b, soft_bucket_loss, prepare_fourier_inputs, use_amp=False)
    out["total"].backward()
    assert ours._core.flat_grad_of(ours) is not None
    before = {n: p.grad.clone() for n, p in ours.named_parameters() if p.grad is not None}
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                            device_id=torch.device("cuda:0"))
    try:
        average_gradients(ours)
        torch.cuda.synchronize()
    finally:
        dist.destroy_process_group()
    for n, p in ours.named_parameters():
        if n in before:
            assert torch.equal(p.grad, before[n]), n
