"""B200-native CTC forced aligner: a drop-in for fast_forced_aligner's API."""
from .alignment import (AlignmentBatch, align, align_packed, emission_validity, load_extension,
                        validate_inputs)

__all__ = ["AlignmentBatch", "align", "align_packed", "emission_validity", "load_extension",
           "validate_inputs"]
