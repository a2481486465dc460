"""Generates tests/golden/finetune_reference.pt by running the reference's own
finetune loss body (chessdecoder/finetune/train.py, the statements inside its
``torch.autocast`` block: Fourier inputs, both passes, board / final-move /
thinking-move / WL / D losses and the weighted total) on a small model.

The statements are taken from the reference source with ``ast`` and executed
as they are, in a namespace that provides what the loop defines before them:
the batch tensors, ``board_ce_fn`` / ``move_ce_fn`` (``nn.CrossEntropyLoss(
ignore_index=-100, reduction='none')``, train.py:179-181), the vocabulary
sizes and ``prepare_fourier_inputs`` / ``soft_bucket_loss`` imported from the
reference (chessdecoder/models/vocab.py, chessdecoder/utils/training.py, both
import without torchtune), and the loss weights of
chessdecoder/finetune/config.yaml.  The reference model itself needs
torchtune, absent here, so the model is the repository's fp32 restatement
(oracle/model.py, pinned separately by backbone_reference.pt); what this
fixture pins is the loss body: masks, gathers, normalisers, weights.

Run where the ChessDecoder repository is mounted, its root given by the
REFERENCE_ROOT environment variable (required):

    REFERENCE_ROOT=<ChessDecoder checkout> python tests/golden/make_finetune_golden.py
"""
from __future__ import annotations

import ast
import os
import sys
from pathlib import Path

import torch
import torch.nn as nn

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

CONFIG = dict(embed_dim=64, num_heads=2, num_layers=1, max_seq_len=512, d_ff=96)
SEED = 3
WEIGHTS = dict(final_move_weight=3.0, thinking_move_weight=3.0, board_weight=1.0, wl_weight=3.0, d_weight=3.0)
BATCH_KEYS = ("input_ids", "board_target_ids", "move_target_ids", "move_mask", "thinking_move_mask", "wl_positions",
              "d_positions", "wl_targets", "d_targets", "wdl_valid", "block_id")


def reference_root() -> Path:
    """The ChessDecoder checkout named by REFERENCE_ROOT (required)."""
    if not os.environ.get("REFERENCE_ROOT"):
        raise SystemExit("set REFERENCE_ROOT to the root of the ChessDecoder repository")
    return Path(os.environ["REFERENCE_ROOT"])


def loss_body_source(train_py: Path) -> ast.Module:
    """The statements inside the ``with torch.autocast(...)`` block of the
    finetune loop, as a module."""
    tree = ast.parse(train_py.read_text())
    for node in ast.walk(tree):
        if isinstance(node, ast.With) and any(
                isinstance(it.context_expr, ast.Call) and ast.unparse(it.context_expr.func) == "torch.autocast"
                for it in node.items):
            mod = ast.Module(body=node.body, type_ignores=[])
            ast.fix_missing_locations(mod)
            return mod
    raise SystemExit("no torch.autocast block found in " + str(train_py))


def main():
    ref = reference_root()
    sys.path.insert(0, str(ref))
    from chessdecoder.models.vocab import board_vocab_size, move_vocab_size, vocab_size
    from chessdecoder.utils.training import prepare_fourier_inputs, soft_bucket_loss
    from chessdecoder_b200 import data
    from oracle.model import OracleChessDecoder

    code = compile(loss_body_source(ref / "chessdecoder/finetune/train.py"), "finetune/train.py:loss_body", "exec")
    torch.manual_seed(SEED)
    model = OracleChessDecoder(vocab_size, **CONFIG)
    batch = data.finetune_batches(1, 2, CONFIG["max_seq_len"], seed=SEED, min_lines=1, max_lines=2, min_depth=1,
                                  max_depth=2)[0]
    batch = {k: batch[k] for k in BATCH_KEYS}
    ns = dict(batch, torch=torch, model=model, device=torch.device("cpu"), IGNORE_INDEX=-100,
              board_ce_fn=nn.CrossEntropyLoss(ignore_index=-100, reduction="none"),
              move_ce_fn=nn.CrossEntropyLoss(ignore_index=-100, reduction="none"),
              board_vocab_size=board_vocab_size, move_vocab_size=move_vocab_size,
              prepare_fourier_inputs=prepare_fourier_inputs, soft_bucket_loss=soft_bucket_loss, **WEIGHTS)
    exec(code, ns)
    ns["total_loss"].backward()
    losses = {n: ns[n].detach().clone() for n in ("final_move_loss", "thinking_move_loss", "board_loss", "wl_loss",
                                                  "d_loss", "total_loss")}
    grads = {n: p.grad.detach().clone() for n, p in model.named_parameters()
             if p.grad is not None and (n.endswith("bias") or n.endswith("scale"))}
    torch.save({"config": CONFIG, "seed": SEED, "weights": WEIGHTS, "batch": batch, "losses": losses, "grads": grads},
               HERE / "finetune_reference.pt")
    print("wrote finetune_reference.pt", {k: round(float(v), 5) for k, v in losses.items()})


if __name__ == "__main__":
    main()
