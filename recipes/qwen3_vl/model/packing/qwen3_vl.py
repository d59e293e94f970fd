"""Packed 3-D (M-RoPE) position ids for Qwen3-VL (reference: recipes/qwen3_vl/model/packing/qwen3_vl.py:8-143).

Position semantics are the model's: inside one packed segment, text tokens
advance all three axes together; the ``t*(h/m)*(w/m)`` placeholder tokens of
an image (the tokens right after a ``<|vision_start|>``) take their
(temporal, row, column) grid coordinates offset by the running position, and
the text after an image resumes at ``max + 1``.  Segments continue from the
previous segment's maximum + 1 (cumulative offsets across the pack), which
does not change attention inside a segment because rotary attention only sees
position differences.

Runs on the host over the collated CPU batch, once per micro-batch, before the
batch is copied to the GPU.
"""

from __future__ import annotations

from typing import Any, Optional

import torch


def _image_starts(ids: torch.Tensor, image_token_id: int, vision_start_id: int) -> torch.Tensor:
    """Indices of image placeholder runs: an image token directly after a vision-start token."""
    vs = (ids[:-1] == vision_start_id) & (ids[1:] == image_token_id)
    return torch.nonzero(vs).flatten() + 1


def _segment_positions(ids: torch.Tensor, grids: Optional[torch.Tensor], starts: torch.Tensor, merge: int,
                       video_token_id: Optional[int]) -> torch.Tensor:
    L = ids.numel()
    if video_token_id is not None and bool((ids == video_token_id).any()):
        raise NotImplementedError("Packed Qwen3-VL training only supports text+image inputs, not video inputs.")
    out = torch.empty(3, L, dtype=torch.long)
    cursor, nxt = 0, 0
    for i, s in enumerate(starts.tolist()):
        t, h, w = (int(x) for x in grids[i])
        gh, gw = h // merge, w // merge
        if s > cursor:
            out[:, cursor:s] = torch.arange(nxt, nxt + s - cursor)
            nxt += s - cursor
        n = t * gh * gw
        if s + n > L:
            raise ValueError("image placeholder run is cut by the segment end")
        tt = torch.arange(t).repeat_interleave(gh * gw)
        hh = torch.arange(gh).repeat_interleave(gw).repeat(t)
        ww = torch.arange(gw).repeat(t * gh)
        out[0, s:s + n] = tt + nxt
        out[1, s:s + n] = hh + nxt
        out[2, s:s + n] = ww + nxt
        nxt += max(t, gh, gw)
        cursor = s + n
    if cursor < L:
        out[:, cursor:] = torch.arange(nxt, nxt + L - cursor)
    return out


def build_qwen3_vl_packed_position_ids(*, input_ids: torch.Tensor, pack_segment_ids: torch.Tensor,
                                       image_grid_thw: Optional[torch.Tensor], model_config: Any) -> torch.Tensor:
    """[3, B, T] position ids for a packed batch; padding (segment 0) keeps position 1 like the reference."""
    if input_ids.ndim != 2:
        raise ValueError(f"Expected 2D input_ids, got shape {tuple(input_ids.shape)}.")
    if pack_segment_ids.shape != input_ids.shape:
        raise ValueError("pack_segment_ids must have the same shape as input_ids, "
                         f"got {tuple(pack_segment_ids.shape)} vs {tuple(input_ids.shape)}.")
    ids_all = input_ids.detach().cpu()
    seg_all = pack_segment_ids.detach().cpu()
    grids = image_grid_thw.detach().cpu().long() if image_grid_thw is not None else None
    B, T = ids_all.shape
    pos = torch.ones(3, B, T, dtype=torch.long)
    img_tok = int(model_config.image_token_id)
    vs_tok = int(model_config.vision_start_token_id)
    vid_tok = getattr(model_config, "video_token_id", None)
    merge = int(model_config.vision_config.spatial_merge_size)
    cursor = 0
    for b in range(B):
        seg = seg_all[b]
        valid = seg > 0
        if not bool(valid.any()):
            continue
        sv = seg[valid]
        change = torch.nonzero(sv[1:] != sv[:-1]).flatten() + 1
        bounds = [0] + change.tolist() + [int(sv.numel())]
        idx = torch.nonzero(valid).flatten()
        nxt = 0
        for a, e in zip(bounds[:-1], bounds[1:]):
            cols = idx[a:e]
            ids = ids_all[b, cols]
            starts = _image_starts(ids, img_tok, vs_tok)
            g = None
            if starts.numel():
                if grids is None:
                    raise ValueError("Packed multimodal samples require image_grid_thw to build position_ids.")
                g = grids[cursor:cursor + starts.numel()]
                if g.shape[0] != starts.numel():
                    raise ValueError("image_grid_thw does not match the number of packed image samples.")
                cursor += starts.numel()
            p = _segment_positions(ids, g, starts, merge, None if vid_tok is None else int(vid_tok)) + nxt
            pos[:, b, cols] = p
            nxt = int(p.max()) + 1
    if grids is not None and cursor != int(grids.shape[0]):
        raise ValueError("Packed image metadata does not align with packed token segments: "
                         f"consumed {cursor}, available {int(grids.shape[0])}.")
    return pos


__all__ = ["build_qwen3_vl_packed_position_ids"]
