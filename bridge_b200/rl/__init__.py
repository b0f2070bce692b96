"""RL objectives over the token tree."""

from .objective import SegmentPPOObjectiveAdapter
