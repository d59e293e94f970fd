"""File sources of the data runtime: jsonl rows are parsed on demand from a byte-offset index and
parquet rows come from one Arrow table, with the same order, sharding and global indices as reading
the whole file; manifests concatenate their files; a changed file is indexed again."""

from __future__ import annotations

import json
import os

import pyarrow as pa
import pyarrow.parquet as pq
import pytest

from mvp_engine.data.runtime import RuntimeContext, _file_source, _open_rows, _read_rows

ROWS = [{"id": i, "text": f"doc {i} é中" + "x" * (i % 7)} for i in range(23)]


def _write_jsonl(path, rows, blank_every=5):
    with open(path, "w", encoding="utf-8") as f:
        for i, r in enumerate(rows):
            f.write(json.dumps(r, ensure_ascii=False) + "\n")
            if i % blank_every == 0:
                f.write("\n   \n")  # blank lines are not rows


def _write_parquet(path, rows):
    pq.write_table(pa.Table.from_pylist(rows), path, row_group_size=4)


def _shards(path, world, shuffle):
    out = []
    for r in range(world):
        ctx = RuntimeContext(seed=7, dp_rank=r, dp_world=world, epoch=1)
        out.append(list(_file_source(str(path), ctx, {"shuffle_mode": "row" if shuffle else "none"})))
    return out


def _expected_order(n, world, shuffle):
    order = list(range(n))
    if shuffle:
        RuntimeContext(seed=7, epoch=1).rng("order").shuffle(order)
    return [order[r::world] for r in range(world)]


@pytest.mark.parametrize("fmt", ["jsonl", "parquet"])
@pytest.mark.parametrize("shuffle", [False, True])
def test_rows_order_and_shards_match_the_whole_file(tmp_path, fmt, shuffle):
    path = tmp_path / f"data.{fmt}"
    (_write_jsonl if fmt == "jsonl" else _write_parquet)(path, ROWS)
    assert _read_rows(str(path)) == ROWS
    shards = _shards(path, 3, shuffle)
    for got, want in zip(shards, _expected_order(len(ROWS), 3, shuffle)):
        assert [r["__global_index__"] for r in got] == want
        assert all({k: v for k, v in r.items() if k != "__global_index__"} == ROWS[r["__global_index__"]]
                   for r in got)
    assert sorted(r["id"] for s in shards for r in s) == list(range(len(ROWS)))


def test_manifest_concatenates_its_files(tmp_path):
    _write_jsonl(tmp_path / "a.jsonl", ROWS[:10])
    _write_parquet(tmp_path / "b.parquet", ROWS[10:])
    (tmp_path / "m.json").write_text(json.dumps({"files": ["a.jsonl", "b.parquet"]}))
    assert _read_rows(str(tmp_path / "m.json")) == ROWS
    got = _shards(tmp_path / "m.json", 2, True)
    for shard in got:
        for r in shard:
            assert r["id"] == r["__global_index__"]


def test_json_list_source(tmp_path):
    (tmp_path / "l.json").write_text(json.dumps(ROWS[:5]))
    assert _read_rows(str(tmp_path / "l.json")) == ROWS[:5]


def test_changed_file_is_indexed_again(tmp_path):
    path = tmp_path / "grow.jsonl"
    _write_jsonl(path, ROWS[:4])
    first = _open_rows(str(path))
    assert len(first) == 4 and _open_rows(str(path)) is first
    with open(path, "a", encoding="utf-8") as f:
        f.write(json.dumps(ROWS[4]) + "\n")
    os.utime(path, ns=(os.stat(path).st_atime_ns, os.stat(path).st_mtime_ns + 1_000_000))
    assert len(_open_rows(str(path))) == 5


def test_jsonl_index_is_offsets_only(tmp_path):
    path = tmp_path / "big.jsonl"
    _write_jsonl(path, ROWS * 10)
    src = _open_rows(str(path))
    assert src.offsets.itemsize == 8 and len(src.offsets) == len(ROWS) * 10
    assert not hasattr(src, "rows")


def test_unknown_suffix_is_refused(tmp_path):
    path = tmp_path / "x.csv"
    path.write_text("a,b\n")
    with pytest.raises(ValueError, match="Unsupported file source"):
        _open_rows(str(path))


def test_lance_source_shards_and_batches_takes(monkeypatch):
    """The lance source against a stand-in module (the package is not installed here): every rank gets
    its slice of the (shuffled) index order, fetched with ``take`` in chunks, with global indices."""
    import sys
    import types

    from mvp_engine.data.runtime import _SOURCES

    takes = []

    class _Table:
        def __init__(self, rows):
            self.rows = rows

        def to_pylist(self):
            return list(self.rows)

    class _Ds:
        def count_rows(self):
            return 600

        def take(self, idx):
            takes.append(len(idx))
            return _Table([{"id": i} for i in idx])

    monkeypatch.setitem(sys.modules, "lance", types.SimpleNamespace(dataset=lambda path: _Ds()))
    source = _SOURCES["lance"]
    seen = []
    for r in range(2):
        ctx = RuntimeContext(seed=7, dp_rank=r, dp_world=2, epoch=1)
        rows = list(source("mem://x", ctx, {"shuffle_mode": "fragment_aware"}))
        assert all(row["id"] == row["__global_index__"] for row in rows)
        assert [row["id"] for row in rows] == _expected_order(600, 2, True)[r]
        seen += [row["id"] for row in rows]
    assert sorted(seen) == list(range(600))
    assert max(takes) <= 256
