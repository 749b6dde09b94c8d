"""B200-native CTC forced aligner: a drop-in for fast_forced_aligner's API."""
from .alignment import (AlignmentBatch, align, align_packed, emission_validity, load_extension, log_softmax,
                        row_logsumexp, token_spans, token_timestamps, validate_inputs)
from .sharding import ShardedAlignment, align_sharded, partition_records, shard_of_rank

__all__ = ["AlignmentBatch", "ShardedAlignment", "align", "align_packed", "align_sharded",
           "emission_validity", "load_extension", "log_softmax", "partition_records", "row_logsumexp",
           "shard_of_rank", "token_spans", "token_timestamps", "validate_inputs"]
