"""The cdk:: custom ops (chessdecoder_b200/ops.py) without a GPU: they are
registered, and a train.py-shaped forward and loss of the drop-in ChessDecoder
(both masks, input_pos, heads, soft_bucket_loss) propagates shapes under
FakeTensorMode with CUDA fake tensors, as does each backward op: every op has
a fake implementation (the shape-only tracing of torch.compile's first stage).
The real backward through the ops' autograd formulas is a GPU test."""
import torch
import torch.nn.functional as F
from torch._subclasses.fake_tensor import FakeTensorMode

SMALL = dict(embed_dim=64, num_heads=2, num_layers=2, max_seq_len=64, d_ff=96)


def test_ops_are_registered():
    import chessdecoder_b200.ops  # noqa: F401
    for name in ("linear", "linear_backward", "soft_bucket_ce", "backbone_fwd", "backbone_bwd_"):
        assert hasattr(torch.ops.cdk, name), name


def test_dropin_forward_loss_backward_under_fake_tensors():
    from chessdecoder_b200.model import ChessDecoder, soft_bucket_loss
    B, S = 2, 64
    with FakeTensorMode():
        with torch.device("cuda"):
            model = ChessDecoder(1968, **SMALL)
        x = torch.randint(0, 1968, (B, S), device="cuda")
        bid = torch.randint(0, 8, (B, S), device="cuda")
        wl_pos = torch.zeros(B, S, dtype=torch.bool, device="cuda")
        vals = torch.zeros(B, S, device="cuda")
        h_c = model(x, mask_type="causal", wl_values=vals, d_values=vals, wl_positions=wl_pos, d_positions=wl_pos)
        h_p = model(x, mask_type="prefix", block_id=bid, wl_values=vals, d_values=vals, wl_positions=wl_pos,
                    d_positions=wl_pos, input_pos=torch.arange(S, device="cuda") + 3)
        assert h_c.shape == (B, S, 64) and h_p.shape == (B, S, 64) and h_p.dtype == torch.float32
        board = model.board_head(h_c)
        moves = model.policy_head(h_p)
        wl = model.wl_head(h_p[:, 0])
        assert board.shape == (B, S, 41) and moves.shape == (B, S, 1924) and wl.shape == (B, 100)
        loss = (F.cross_entropy(board.reshape(-1, 41), x.reshape(-1) % 41)
                + F.cross_entropy(moves.reshape(-1, 1924), x.reshape(-1))
                + soft_bucket_loss(wl, vals[:, 0], model.wl_bucket_centers, torch.ones(B, dtype=torch.bool,
                                                                                       device="cuda")))
        assert loss.shape == ()
        # the backward ops' fake implementations (autograd itself needs a real
        # CUDA device for CUDA tensors; the GPU tests run the real backward)
        dx, dw, db = torch.ops.cdk.linear_backward(torch.empty_like(moves), h_p, model.policy_head.weight)
        assert dx.shape == h_p.shape and dw.shape == (1924, 64) and db.shape == (1924,)
        from chessdecoder_b200.engine import flat_layout
        _, numel = flat_layout(model.cfg)
        out = torch.ops.cdk.backbone_fwd(x, None, None, None, None, None, None, model._op_id, model._backbone_params())
        torch.ops.cdk.backbone_bwd_(out[1], torch.empty_like(out[0]), torch.zeros(numel, device="cuda"))
