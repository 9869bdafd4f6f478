"""Candidate-segment layout: several GR candidates over one shared history.

The reference serves a GR request by packing every candidate into one suffix
(worker/prompt.py:24-55), so a candidate also attends to the candidates
packed before it. Here each candidate can instead see only the user's
history and its own suffix. The path keeps working in one coordinate system,
called segment positions:

* positions below ``start`` (the history rounded down to a block boundary)
  are history, shared by all candidates;
* candidate ``c``'s token with true position ``start + i`` sits at segment
  position ``start + c * tokens + i``; ``tokens`` is a whole number of blocks
  holding the history tail past ``start`` (fewer than BS tokens, copied into
  every segment) followed by the candidate's suffix. It is sized for the
  longest tail (BS - 1), so every user with the same suffix length gets the
  same segment stride, and buffers (and planner workspaces) of users with
  different history lengths have the same shapes;
* a row of candidate ``c`` never sees segments other than its own (the
  attention and selection kernels skip them; the planner never sees them
  because no row selects them).

Block ids, summaries, window records and each fetch's current KV use segment
positions, so the fetch planner needs no change: history blocks deduplicate
across candidates (one fetch per block however many candidates select it)
and suffix blocks stay private to their candidate. With one candidate the
layout is not used and the path is exactly the reference's.
"""

from dataclasses import dataclass


@dataclass(frozen=True)
class SegmentLayout:
    history: int        # true history length (tokens already cached)
    extend: int         # suffix tokens per candidate
    candidates: int
    block_size: int

    def __post_init__(self):
        bs = self.block_size
        if bs < 1 or bs & (bs - 1):
            raise ValueError("block_size must be a power of two")
        if self.history < 0 or self.extend < 1 or self.candidates < 1:
            raise ValueError("history >= 0, extend >= 1 and candidates >= 1 required")

    @property
    def tail(self):
        """History tokens past the last block boundary (carried into each segment)."""
        return self.history % self.block_size

    @property
    def start(self):
        """First segment position: the history rounded down to a block boundary."""
        return self.history - self.tail

    @property
    def tokens(self):
        """Segment length: the longest tail (BS - 1) + suffix, in whole blocks."""
        bs = self.block_size
        return -(-(bs - 1 + self.extend) // bs) * bs

    @property
    def blocks(self):
        return self.tokens // self.block_size

    @property
    def total(self):
        """True history + suffix length of one candidate."""
        return self.history + self.extend

    def segments(self):
        """(segment_start, segment_tokens) as the C ABI takes them."""
        return (self.start, self.tokens)

    def position(self, candidate, index):
        """Segment position of suffix token ``index`` of ``candidate``."""
        return self.start + candidate * self.tokens + self.tail + index

    def positions(self):
        """Segment positions of all rows, candidate-major (row = c * extend + i)."""
        return [self.position(c, i) for c in range(self.candidates) for i in range(self.extend)]

    def true_position(self, position):
        """True position of a segment position (history positions map to themselves)."""
        if position < self.start:
            return position
        return self.start + (position - self.start) % self.tokens

    def candidate_of(self, position):
        """Candidate owning a segment position, or None for shared history."""
        if position < self.start:
            return None
        return (position - self.start) // self.tokens

    def true_block(self, block):
        """True block id of a segment block id (history blocks map to themselves)."""
        return self.true_position(block * self.block_size) // self.block_size

    def segment_block(self, candidate, block):
        """Segment block id of a candidate's true block id."""
        first = self.start // self.block_size
        if block < first:
            return block
        return first + candidate * self.blocks + (block - first)
