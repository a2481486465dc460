"""ORACLE (test infrastructure only): the reference training step restated in fp32.

Follows chessdecoder/train/train.py:157-253 with use_amp disabled:
prepare_fourier_inputs (utils/training.py:114-133) -> pass 1 (causal) ->
board head + masked CE (:180-194) -> pass 2 (prefix) -> policy head + masked
CE (:204-207) -> WL head at stm+1 (:210-222) -> D head at WL positions
(:225-233) -> total loss (:236-241) -> backward -> clip_grad_norm_(10) ->
AdamW step (:248-253).  ``soft_bucket_loss`` restates utils/training.py:24-50.
Both helpers are pinned against the reference's own functions by
tests/golden/utils_reference.pt.  ``finetune_step_losses`` restates the
finetune step's loss (chessdecoder/finetune/train.py:272-355) the same way.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

IGNORE_INDEX = -100


def soft_bucket_loss(logits, target_values, bucket_centers, valid_mask):
    N = target_values.shape[0]
    nb = bucket_centers.shape[0]
    if N == 0 or valid_mask.sum() == 0:
        return torch.tensor(0.0, device=logits.device)
    diffs = target_values.unsqueeze(-1) - bucket_centers
    lower = ((diffs >= 0).long().sum(dim=-1) - 1).clamp(0, nb - 2)
    upper = lower + 1
    lc, uc = bucket_centers[lower], bucket_centers[upper]
    w_up = ((target_values - lc) / (uc - lc).clamp(min=1e-8)).clamp(0.0, 1.0)
    soft = torch.zeros(N, nb, device=logits.device)
    soft.scatter_(1, lower.unsqueeze(1), (1 - w_up).unsqueeze(1))
    soft.scatter_(1, upper.unsqueeze(1), w_up.unsqueeze(1))
    loss = -(soft * F.log_softmax(logits, dim=-1)).sum(dim=-1)
    return (loss * valid_mask.float()).sum() / (valid_mask.sum() + 1e-8)


def prepare_fourier_inputs(model, wl_targets, d_targets, wl_positions, d_positions):
    wl_in = torch.zeros_like(wl_targets)
    d_in = torch.zeros_like(d_targets)
    if wl_positions.any():
        wl_in[wl_positions] = model.discretize_to_bucket(wl_targets[wl_positions], model.wl_bucket_centers)
    if d_positions.any():
        d_in[d_positions] = model.discretize_to_bucket(d_targets[d_positions], model.d_bucket_centers)
    return wl_in, d_in


def step_losses(model, batch, weights=(5.0, 1.0, 1.0, 1.0)):
    """Forward of one training step; returns a dict of losses and argmax predictions."""
    move_w, board_w, wl_w, d_w = weights
    dev = next(model.parameters()).device
    b = {k: v.to(dev) for k, v in batch.items()}
    input_ids, board_t, move_t = b["input_ids"], b["board_target_ids"], b["move_target_ids"]
    move_mask, wl_pos, d_pos = b["move_mask"], b["wl_positions"], b["d_positions"]
    wl_t, d_t, wdl_valid, block_id = b["wl_targets"], b["d_targets"], b["wdl_valid"], b["block_id"]
    ce = nn.CrossEntropyLoss(ignore_index=IGNORE_INDEX, reduction="none")

    wl_in, d_in = prepare_fourier_inputs(model, wl_t, d_t, wl_pos, d_pos)
    h_causal = model(input_ids, mask_type="causal", wl_values=wl_in, d_values=d_in, wl_positions=wl_pos,
                     d_positions=d_pos)
    board_logits = model.board_head(h_causal)
    board_mask = board_t != IGNORE_INDEX
    first_move = move_mask.int().argmax(dim=1)
    has_moves = move_mask.any(dim=1)
    first_move[~has_moves] = move_mask.size(1)
    idx = torch.arange(move_mask.size(1), device=dev).unsqueeze(0)
    board_mask = board_mask & ~(idx < first_move.unsqueeze(1))
    ce_board = ce(board_logits.view(-1, board_logits.shape[-1]), board_t.view(-1)).view(board_t.shape)
    board_loss = (ce_board * board_mask.float()).sum() / (board_mask.sum() + 1e-8)

    h_prefix = model(input_ids, mask_type="prefix", block_id=block_id, wl_values=wl_in, d_values=d_in,
                     wl_positions=wl_pos, d_positions=d_pos)
    move_logits = model.policy_head(h_prefix)
    ce_move = ce(move_logits.view(-1, move_logits.shape[-1]), move_t.view(-1)).view(move_t.shape)
    move_loss = (ce_move * move_mask.float()).sum() / (move_mask.sum() + 1e-8)

    nz = move_mask.nonzero(as_tuple=False)
    wl_logits = d_logits = None
    if nz.shape[0] > 0:
        seq = (nz[:, 1] + 1).clamp(max=h_prefix.shape[1] - 1)
        wl_logits = model.wl_head(h_prefix[nz[:, 0], seq])
        wl_loss = soft_bucket_loss(wl_logits, wl_t[move_mask], model.wl_bucket_centers, wdl_valid[move_mask])
    else:
        wl_loss = torch.tensor(0.0, device=dev)
    if wl_pos.any():
        d_logits = model.d_head(h_prefix[wl_pos])
        d_loss = soft_bucket_loss(d_logits, d_t[d_pos], model.d_bucket_centers, wdl_valid[d_pos])
    else:
        d_loss = torch.tensor(0.0, device=dev)
    total = move_w * move_loss + board_w * board_loss + wl_w * wl_loss + d_w * d_loss
    return {
        "total": total, "move": move_loss, "board": board_loss, "wl": wl_loss, "d": d_loss,
        "board_argmax": board_logits.argmax(-1), "board_mask": board_mask, "board_logits": board_logits,
        "move_argmax": move_logits.argmax(-1), "move_mask": move_mask, "move_logits": move_logits,
        "wl_argmax": None if wl_logits is None else wl_logits.argmax(-1),
        "d_argmax": None if d_logits is None else d_logits.argmax(-1),
    }


def finetune_step_losses(model, batch, weights=(3.0, 1.0, 3.0, 3.0, 3.0)):
    """Forward of one finetune step (chessdecoder/finetune/train.py:272-355,
    use_amp off): the board mask starts at the first move of either kind
    (:287-299), the policy head is scored at ``move_mask`` rows (:309-312),
    the thinking head at ``thinking_move_mask`` rows with the same targets
    (:315-318), the WL head at stm+1 of every move row of either kind
    (:321-335), the D head at WL positions (:337-346).  weights = (final move,
    board, wl, d, thinking move) as in chessdecoder/finetune/config.yaml."""
    final_w, board_w, wl_w, d_w, think_w = weights
    dev = next(model.parameters()).device
    b = {k: v.to(dev) for k, v in batch.items()}
    input_ids, board_t, move_t = b["input_ids"], b["board_target_ids"], b["move_target_ids"]
    move_mask, think_mask = b["move_mask"], b["thinking_move_mask"]
    wl_pos, d_pos = b["wl_positions"], b["d_positions"]
    wl_t, d_t, wdl_valid, block_id = b["wl_targets"], b["d_targets"], b["wdl_valid"], b["block_id"]
    ce = nn.CrossEntropyLoss(ignore_index=IGNORE_INDEX, reduction="none")

    wl_in, d_in = prepare_fourier_inputs(model, wl_t, d_t, wl_pos, d_pos)
    h_causal = model(input_ids, mask_type="causal", wl_values=wl_in, d_values=d_in, wl_positions=wl_pos,
                     d_positions=d_pos)
    board_logits = model.board_head(h_causal)
    board_mask = board_t != IGNORE_INDEX
    any_move = move_mask | think_mask
    first_move = any_move.int().argmax(dim=1)
    first_move[~any_move.any(dim=1)] = any_move.size(1)
    idx = torch.arange(any_move.size(1), device=dev).unsqueeze(0)
    board_mask = board_mask & ~(idx < first_move.unsqueeze(1))
    ce_board = ce(board_logits.view(-1, board_logits.shape[-1]), board_t.view(-1)).view(board_t.shape)
    board_loss = (ce_board * board_mask.float()).sum() / (board_mask.sum() + 1e-8)

    h_prefix = model(input_ids, mask_type="prefix", block_id=block_id, wl_values=wl_in, d_values=d_in,
                     wl_positions=wl_pos, d_positions=d_pos)
    final_logits = model.policy_head(h_prefix)
    ce_final = ce(final_logits.view(-1, final_logits.shape[-1]), move_t.view(-1)).view(move_t.shape)
    final_loss = (ce_final * move_mask.float()).sum() / (move_mask.sum() + 1e-8)
    think_logits = model.thinking_policy_head(h_prefix)
    ce_think = ce(think_logits.view(-1, think_logits.shape[-1]), move_t.view(-1)).view(move_t.shape)
    think_loss = (ce_think * think_mask.float()).sum() / (think_mask.sum() + 1e-8)

    nz = any_move.nonzero(as_tuple=False)
    if nz.shape[0] > 0:
        seq = (nz[:, 1] + 1).clamp(max=h_prefix.shape[1] - 1)
        wl_logits = model.wl_head(h_prefix[nz[:, 0], seq])
        wl_loss = soft_bucket_loss(wl_logits, wl_t[any_move], model.wl_bucket_centers, wdl_valid[any_move])
    else:
        wl_loss = torch.tensor(0.0, device=dev)
    if wl_pos.any():
        d_logits = model.d_head(h_prefix[wl_pos])
        d_loss = soft_bucket_loss(d_logits, d_t[d_pos], model.d_bucket_centers, wdl_valid[d_pos])
    else:
        d_loss = torch.tensor(0.0, device=dev)
    total = final_w * final_loss + think_w * think_loss + board_w * board_loss + wl_w * wl_loss + d_w * d_loss
    return {"total": total, "move": final_loss, "board": board_loss, "wl": wl_loss, "d": d_loss,
            "think": think_loss, "move_argmax": final_logits.argmax(-1), "think_argmax": think_logits.argmax(-1)}


def train_step(model, optimizer, batch, max_norm=10.0, weights=(5.0, 1.0, 1.0, 1.0)):
    """One full optimizer step (grad_accum 1); returns the forward's loss dict."""
    optimizer.zero_grad(set_to_none=True)
    out = step_losses(model, batch, weights)
    out["total"].backward()
    torch.nn.utils.clip_grad_norm_(model.parameters(), max_norm=max_norm)
    optimizer.step()
    return out
