"""Data runtime, packing invariants, collation and varlen metadata (CPU)."""

import torch

from mvp_engine.data import Dataset, RuntimeContext, SyntheticTokenizer
from mvp_engine.kit.llm.data import (LLMBatchCollator, LLMDataKit, LLMDataSpec, LLMLoaderSpec, LLMPackingAssembler,
                                     LLMPackingSpec, LLMPretrainTextTokenizationHandler, LLMSample, LLMSampleSpec,
                                     LLMSourceSpec, LLMTokenIdsSchemaHandler, varlen_metadata)


def _spec(max_len=64, isolate=True, tail="drop", bs=2):
    tok = SyntheticTokenizer(vocab_size=1000)
    sample = LLMSampleSpec(LLMTokenIdsSchemaHandler(), LLMPretrainTextTokenizationHandler(tok, max_seq_len=max_len,
                                                                                            add_eos=False))
    return LLMDataSpec(source=LLMSourceSpec("synthetic://text?vocab=1000&min_len=5&max_len=40&num_rows=50",
                                            dataset_source="synthetic_text", resample=False, shuffle_mode="none"),
                       sample=sample,
                       packing=LLMPackingSpec(max_len, tail_policy=tail, isolate_attention=isolate,
                                              isolate_position_ids=isolate),
                       loader=LLMLoaderSpec(batch_size=bs))


def test_packing_invariants():
    kit = LLMDataKit()
    spec = _spec()
    packs = list(kit.build_dataset(spec))
    assert packs
    for p in packs:
        n = p["input_ids"].numel()
        assert n == 64
        seg = p["pack_segment_ids"]
        assert seg[0] == 1 and bool((seg[1:] - seg[:-1] >= 0).all())
        pos = p["position_ids"]
        starts = torch.nonzero(torch.diff(seg)).reshape(-1) + 1
        assert int(pos[0]) == 0 and all(int(pos[s]) == 0 for s in starts)


def test_pack_pad_tail_and_resume():
    tok = SyntheticTokenizer(vocab_size=100)
    handler = LLMPretrainTextTokenizationHandler(tok, max_seq_len=100, add_eos=False)
    sspec = LLMSampleSpec(LLMTokenIdsSchemaHandler(), handler)
    asm = LLMPackingAssembler(LLMPackingSpec(10, tail_policy="pad", isolate_attention=True))
    out = []
    for n in (4, 9, 3):
        out += asm.push(LLMSample.from_row({"input_ids": list(range(1, n + 1))}, sample_spec=sspec))
    state = asm.state_dict()
    asm2 = LLMPackingAssembler(LLMPackingSpec(10, tail_policy="pad", isolate_attention=True))
    asm2.load_state_dict(state)
    tail = asm2.finish()
    assert len(out) == 1 and len(tail) == 1
    t = tail[0]
    assert t.attention_mask.count(0) == 4 and t.labels[-1] == -100 and t.input_ids[-1] == tok.pad_token_id
    assert asm.fingerprint() == asm2.fingerprint()


def test_collator_counts_and_varlen():
    seg = torch.tensor([[1, 1, 1, 2, 2, 0], [1, 1, 1, 1, 1, 1]])
    batch = []
    for row in seg:
        n = row.numel()
        batch.append({"input_ids": torch.arange(n), "attention_mask": (row > 0).long(),
                      "labels": torch.where(row > 0, torch.arange(n), torch.full((n,), -100)),
                      "pack_segment_ids": row, "source_sample_num": int(row.max())})
    out = LLMBatchCollator(pad_token_id=0)(batch)
    assert out["total_tokens"] == 11
    # shifted labels: last token of each row is ignored; padding ignored
    assert out["effective_tokens"] == 4 + 5
    cu, mx, pos = varlen_metadata(seg)
    assert cu.tolist() == [0, 3, 5, 6, 12] and mx == 6
    assert pos[0].tolist() == [0, 1, 2, 0, 1, 0]
    assert out["attention_token_pairs"] == 9 + 4 + 36


def test_rank_sharding_disjoint():
    seen = []
    for r in range(2):
        ctx = RuntimeContext(seed=1, dp_rank=r, dp_world=2)
        rows = list(Dataset.from_source("synthetic_text", "synthetic://text?num_rows=10&min_len=1&max_len=2",
                                        context=ctx))
        seen.append({row["id"] for row in rows})
    assert seen[0].isdisjoint(seen[1]) and len(seen[0] | seen[1]) == 10


def test_dataloader_batches():
    kit = LLMDataKit()
    spec = _spec(bs=2)
    loader = kit.build_dataloader(kit.build_dataset(spec), spec)
    b = next(iter(loader))
    assert b["input_ids"].shape == (2, 64) and "cu_seq_lens_q" in b and b["cu_seq_lens_q"][-1] == 128


def test_dataloader_position_resumes_the_stream():
    """A loader restored from ``state_dict`` continues with the batch after the last one handed out."""
    kit = LLMDataKit()
    spec = _spec(bs=2)
    first = kit.build_dataloader(kit.build_dataset(spec), spec)
    it = iter(first)
    seen = [next(it) for _ in range(3)]
    state = first.state_dict()
    assert state == {"batches_into_pass": 3}
    expected = next(it)
    again = kit.build_dataloader(kit.build_dataset(spec), spec)
    again.load_state_dict(state)
    got = next(iter(again))
    assert torch.equal(got["input_ids"], expected["input_ids"])
    assert not torch.equal(got["input_ids"], seen[-1]["input_ids"])


def test_qwen3_recipe_packing_helpers_match_a_direct_construction():
    """Positions restart per document (0 on padding); cu_seqlens list every document of every row, the
    padding suffix being one more; malformed padding is rejected."""
    import pytest
    import torch

    from recipes.qwen3.model.packing import build_packed_fa2_varlen_kwargs, build_packed_text_position_ids

    seg = torch.tensor([[1, 1, 1, 2, 2, 0, 0], [1, 2, 2, 2, 3, 3, 3]])
    pos = build_packed_text_position_ids(torch.zeros_like(seg), seg)
    assert pos.tolist() == [[0, 1, 2, 0, 1, 0, 0], [0, 0, 1, 2, 0, 1, 2]]
    kw = build_packed_fa2_varlen_kwargs(seg)
    assert kw["cu_seq_lens_q"].tolist() == [0, 3, 5, 7, 8, 11, 14] and kw["cu_seq_lens_q"].dtype == torch.int32
    assert kw["max_length_q"] == kw["max_length_k"] == 3 and kw["cu_seq_lens_k"] is kw["cu_seq_lens_q"]
    with pytest.raises(ValueError):
        build_packed_fa2_varlen_kwargs(torch.tensor([[1, 0, 1]]))
    with pytest.raises(ValueError):
        build_packed_fa2_varlen_kwargs(torch.tensor([1, 1]))
