from .c4 import load_c4_documents, load_documents, save_documents
from .sharding import ShardedCorpus, assign_paths, chunk_documents, pack_sequences
from .spec import (
    SpecCorpus, c4_source, fit_routing_from_source, iter_spec_documents, kmeans_routing,
    make_shard_spec, materialize_shard, round_robin_routing, spec_fingerprint,
    synthetic_documents, synthetic_source, verify_routing,
)
from .streaming import ShardCache, ingest_c4_shard, shard_stream, stream_c4_documents, stream_documents
from .synthetic import zipf_documents
from .text import load_tokenizer, split_documents, tokenize_documents, tokenize_one, train_tokenizer

__all__ = [
    "ShardedCorpus", "SpecCorpus", "make_shard_spec", "materialize_shard", "spec_fingerprint",
    "synthetic_documents", "synthetic_source", "c4_source", "kmeans_routing",
    "round_robin_routing", "fit_routing_from_source", "verify_routing", "iter_spec_documents",
    "assign_paths", "pack_sequences", "chunk_documents", "tokenize_documents", "tokenize_one",
    "load_tokenizer", "train_tokenizer", "split_documents", "load_c4_documents", "load_documents",
    "save_documents", "shard_stream", "stream_documents", "stream_c4_documents", "ShardCache",
    "ingest_c4_shard", "zipf_documents",
]
