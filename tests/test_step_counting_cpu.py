"""Step counting / estimation kits and the text tokenisation handler, on CPU (gloo ranks where the
kit reduces across ranks)."""

from __future__ import annotations

import math

import pytest

from mvp_engine.kit.llm.data.tokenization import LLMTokenizationHandler
from mvp_engine.kit.llm.data.types import LLMSegment
from mvp_engine.kit.llm.utils.step_estimation import LLMStepEstimationKit
from mvp_engine.kit.util.step_counting import StepCountingKit, samples_per_step


class _Stream:
    """A finite dataset with the runtime's ``consume(factory)`` contract."""

    def __init__(self, items):
        self.items = list(items)

    def consume(self, factory):
        consumer = factory(None)
        for item in self.items:
            if consumer.push(item) is False:
                break
        return consumer.finish()


def test_single_process_count_rounds_up():
    kit = StepCountingKit()
    r = kit.count_total_steps(_Stream(range(23)), batch_size=2, gradient_accumulation_steps=3,
                              data_parallel_world_size=1)
    assert (r.total_samples, r.samples_per_step, r.total_steps) == (23, 6, 4)
    weighted = StepCountingKit(sample_counter=lambda item: 2)  # e.g. two samples per record
    assert weighted.count_total_steps(_Stream(range(5)), batch_size=1, gradient_accumulation_steps=1,
                                      data_parallel_world_size=1).total_steps == 10


def test_rejects_bad_inputs():
    with pytest.raises(ValueError):
        samples_per_step(0, 1)
    with pytest.raises(RuntimeError):
        StepCountingKit().count_total_steps(_Stream([]), batch_size=1, gradient_accumulation_steps=1,
                                            data_parallel_world_size=1)
    with pytest.raises(TypeError):
        StepCountingKit().count_total_steps([1, 2], batch_size=1, gradient_accumulation_steps=1,
                                            data_parallel_world_size=1)


def _ranks_worker(rank, world, port, sizes):
    import torch.distributed as dist

    from mvp_engine.distributed.init import initialize_process_group

    initialize_process_group()
    kit = LLMStepEstimationKit()
    try:
        r = kit.estimate_total_steps(_Stream(range(sizes[rank])), batch_size=2, gradient_accumulation_steps=2,
                                     data_parallel_world_size=world, data_parallel_group=dist.group.WORLD)
        return ("ok", r.total_steps, r.total_packed_samples, r.samples_per_step)
    except RuntimeError as exc:
        return ("err", str(exc))


def test_ranks_agree_on_the_longest_rank():
    """Every rank gets the same step count: the slowest rank's (ceil of its samples / samples per step),
    with samples summed over ranks."""
    from mvp_engine.testing.utils import spawn_workers

    sizes = (9, 14)
    out = spawn_workers(_ranks_worker, 2, sizes, timeout=300)
    want = max(math.ceil(n / 4) for n in sizes)
    assert out == [("ok", want, sum(sizes), 4)] * 2


def test_an_empty_rank_is_an_error_on_every_rank():
    from mvp_engine.testing.utils import spawn_workers

    out = spawn_workers(_ranks_worker, 2, (5, 0), timeout=300)
    assert [o[0] for o in out] == ["err", "err"] and "no training samples" in out[0][1]


class _Tok:
    eos_token_id = 99

    def __call__(self, text, add_special_tokens=False):
        assert add_special_tokens is False
        return {"input_ids": [ord(c) - 96 for c in text]}  # 'a' -> 1, 'b' -> 2, ...


def test_tokenization_masks_unsupervised_segments_and_closes_with_eos():
    h = LLMTokenizationHandler(tokenizer=_Tok(), max_seq_len=100)
    [(ids, labels, mask)] = h.tokenize([LLMSegment("text", False, "ab"), LLMSegment("text", True, "cd")])
    assert ids == [1, 2, 3, 4, 99] and labels == [-100, -100, 3, 4, 99] and mask == [1] * 5
    [(ids, labels, _)] = h.tokenize([LLMSegment("text", True, "ab"), LLMSegment("tokens", False, [7, 8])])
    assert ids == [1, 2, 7, 8, 99] and labels == [1, 2, -100, -100, -100]  # EOS follows the last segment's loss


def test_tokenization_cuts_max_length_chunks():
    h = LLMTokenizationHandler(tokenizer=_Tok(), max_seq_len=4)
    chunks = h.tokenize([LLMSegment("tokens", True, list(range(1, 10)))])
    assert [c[0] for c in chunks] == [[1, 2, 3, 4], [5, 6, 7, 8], [9, 99]]
    assert all(len(c[0]) == len(c[1]) == len(c[2]) for c in chunks)
    assert LLMTokenizationHandler(tokenizer=_Tok(), max_seq_len=4, add_eos=False).tokenize([]) == []
