"""Synthetic sources and a tokenizer stand-in for offline runs.

``synthetic_text`` rows carry pre-tokenised ``input_ids`` (uniform over the
vocabulary) with document lengths uniform in ``[min_len, max_len]``: the data
of the dense-decoder benchmark configurations.  ``synthetic_mm`` rows carry 1-4
images whose height and width are multiples of 32 in ``[min_px, max_px]``
(pixels drawn N(0, 1) when loaded) interleaved with uniform text tokens, with
``loss_fraction`` of the text supervised: the data of the VLM SFT
configuration.  Paths look like ``synthetic://text?vocab=151936&min_len=256``;
query parameters override the keyword options of ``Dataset.from_source``.

``SyntheticTokenizer`` provides the attributes the kits read from a Hugging
Face tokenizer (pad/eos ids, special-token lookup, ``__call__`` on text) with a
deterministic hashing encoder, so the same pipelines run with no tokenizer
files on disk.
"""

from __future__ import annotations

import hashlib
from typing import Any, Iterator
from urllib.parse import parse_qs, urlparse

from .runtime import RuntimeContext, register_source

QWEN_SPECIAL_TOKENS = {
    "<|endoftext|>": 151643,
    "<|im_start|>": 151644,
    "<|im_end|>": 151645,
    "<|vision_start|>": 151652,
    "<|vision_end|>": 151653,
    "<|image_pad|>": 151655,
    "<|video_pad|>": 151656,
}


def _opts(path: str, opts: dict) -> dict:
    parsed = urlparse(path)
    merged = dict(opts)
    for k, v in parse_qs(parsed.query).items():
        val: Any = v[-1]
        for cast in (int, float):
            try:
                val = cast(val)
                break
            except ValueError:
                continue
        merged[k] = val
    return merged


@register_source("synthetic_text")
def synthetic_text(path: str, ctx: RuntimeContext, opts: dict) -> Iterator[dict]:
    o = _opts(path, opts)
    vocab = int(o.get("vocab", 151936))
    lo, hi = int(o.get("min_len", 256)), int(o.get("max_len", 4096))
    num_rows = int(o.get("num_rows", 1 << 62))
    rng = ctx.rng("synthetic_text")
    for i in range(ctx.shard_index, num_rows, ctx.num_shards):
        n = rng.randint(lo, hi)
        ids = [rng.randrange(vocab) for _ in range(n)]
        yield {"id": i, "input_ids": ids}


@register_source("synthetic_mm")
def synthetic_mm(path: str, ctx: RuntimeContext, opts: dict) -> Iterator[dict]:
    o = _opts(path, opts)
    vocab = int(o.get("vocab", 151643))  # plain-text ids stay below the special tokens
    min_px, max_px = int(o.get("min_px", 448)), int(o.get("max_px", 1344))
    min_img, max_img = int(o.get("min_images", 1)), int(o.get("max_images", 4))
    text_lo, text_hi = int(o.get("min_text", 64)), int(o.get("max_text", 1024))
    loss_fraction = float(o.get("loss_fraction", 0.3))
    num_rows = int(o.get("num_rows", 1 << 62))
    rng = ctx.rng("synthetic_mm")
    steps = list(range(min_px // 32, max_px // 32 + 1))
    for i in range(ctx.shard_index, num_rows, ctx.num_shards):
        n_img = rng.randint(min_img, max_img)
        images = [{"height": 32 * rng.choice(steps), "width": 32 * rng.choice(steps),
                   "seed": rng.randrange(1 << 31)} for _ in range(n_img)]
        segments = []
        for j in range(n_img + 1):
            n = rng.randint(text_lo, text_hi) // (n_img + 1) + 1
            segments.append([rng.randrange(vocab) for _ in range(n)])
        yield {"id": i, "images": images, "text_segments": segments, "loss_fraction": loss_fraction}


class SyntheticTokenizer:
    """Deterministic stand-in for a Qwen tokenizer (no files needed)."""

    def __init__(self, vocab_size: int = 151936, pad_token_id: int = 151643, eos_token_id: int = 151643,
                 special_tokens: dict[str, int] | None = None) -> None:
        self.vocab_size = vocab_size
        self.pad_token_id = pad_token_id
        self.eos_token_id = eos_token_id
        self.special = dict(QWEN_SPECIAL_TOKENS if special_tokens is None else special_tokens)
        self.pad_token = "<|endoftext|>"
        self.eos_token = "<|endoftext|>"
        self.padding_side = "right"

    def _encode_word(self, w: str) -> int:
        if w in self.special:
            return self.special[w]
        h = int(hashlib.blake2b(w.encode(), digest_size=8).hexdigest(), 16)
        return h % min(self.vocab_size, 151643)

    def encode(self, text: str, add_special_tokens: bool = False) -> list[int]:
        out: list[int] = []
        for tok in text.replace("<|", " <|").replace("|>", "|> ").split():
            out.append(self._encode_word(tok))
        return out

    def __call__(self, text: str, add_special_tokens: bool = False, **_: Any) -> dict[str, list[int]]:
        return {"input_ids": self.encode(text, add_special_tokens)}

    def convert_tokens_to_ids(self, token: str) -> int:
        return self._encode_word(token)

    def __len__(self) -> int:
        return self.vocab_size
