"""Resumable sharded ingestion (data/streaming.py) on an in-memory stream with a toy
tokenizer: the workers of a partition read every item once, a crash after a flush
resumes exactly where the flush left off, and the cache file is the reference's."""

import torch

from opendipaco_b200.data.streaming import ShardCache, ingest_c4_shard, shard_stream, stream_documents


class ByteTokenizer:
    eos_token_id = 0

    def encode(self, text, add_special_tokens=False):
        return [b + 1 for b in text.encode()]


class SkippableRows(list):
    """A list that, like a streaming dataset, can skip a prefix without reading it."""

    skipped_reads = 0

    def skip(self, n):
        return iter(self[n:])


ROWS = SkippableRows({"text": f"doc {i} " + "x" * (i % 5)} for i in range(40))


def test_round_robin_partition_covers_the_stream_once():
    seen = []
    for sid in range(3):
        seen += [i for i, _ in shard_stream(ROWS, num_shards=3, shard_id=sid)]
    assert sorted(seen) == list(range(40))
    assert [i for i, _ in shard_stream(ROWS, num_shards=3, shard_id=1, start_index=10)][:3] == [10, 13, 16]


def test_limit_and_min_tokens():
    tok = ByteTokenizer()
    got = list(stream_documents(ROWS, tok, limit=4, min_doc_tokens=8))
    assert len(got) == 4 and all(len(d) >= 8 for _, d in got)
    assert all(int(d[-1]) == 0 for _, d in got)  # eos appended


def test_crash_after_flush_resumes_exactly(tmp_path):
    tok = ByteTokenizer()
    whole = ingest_c4_shard(tmp_path / "a", shard_id=1, num_shards=2, target_docs=12, tokenizer=tok, source=ROWS,
                            flush_every=3)

    class Crash(Exception):
        pass

    calls = []

    def crash_after_second_flush(count, next_index):
        calls.append((count, next_index))
        if len(calls) == 2:
            raise Crash

    try:
        ingest_c4_shard(tmp_path / "b", shard_id=1, num_shards=2, target_docs=12, tokenizer=tok, source=ROWS,
                        flush_every=3, progress=crash_after_second_flush)
    except Crash:
        pass
    docs, nxt = ShardCache(tmp_path / "b", shard_id=1, num_shards=2).load()
    assert len(docs) == 6 and nxt == calls[-1][1] and nxt % 2 == 0
    resumed = ingest_c4_shard(tmp_path / "b", shard_id=1, num_shards=2, target_docs=12, tokenizer=tok, source=ROWS,
                              flush_every=3)
    assert len(resumed) == 12 and all(torch.equal(x, y) for x, y in zip(whole, resumed))
    blob = torch.load(tmp_path / "b" / "shard_00001_of_00002.pt", weights_only=True)
    assert set(blob) == {"docs", "next_index", "count"} and blob["count"] == 12


def test_cache_is_shared_with_reference(tmp_path, reference_pkg):
    from opendipaco.data.streaming import ShardCache as RefCache

    tok = ByteTokenizer()
    ingest_c4_shard(tmp_path, shard_id=0, num_shards=4, target_docs=5, tokenizer=tok, source=ROWS, flush_every=2)
    docs, nxt = RefCache(tmp_path, shard_id=0, num_shards=4).load()
    ours, ours_next = ShardCache(tmp_path, shard_id=0, num_shards=4).load()
    assert nxt == ours_next and len(docs) == len(ours) == 5
