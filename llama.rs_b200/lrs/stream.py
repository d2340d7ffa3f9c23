"""Incremental UTF-8 output of sampled tokens, per row of a batch (host side).

rust-llama prints a token's bytes only once they form complete UTF-8: `ByteStream`
(main.rs:829-867) and the generation core of the server (server.rs:186-213) append each token's
bytes to a pending buffer, emit its longest valid UTF-8 prefix (Rust's `valid_up_to`) and keep
the rest; at the end the remainder is emitted lossily (`String::from_utf8_lossy`: one U+FFFD per
maximal ill-formed subsequence).  A byte sequence that is invalid (not merely incomplete) stays
pending until that final flush, as in the reference.  `ByteStreams` keeps one such buffer per row
of a batched loop; the token -> bytes table is the caller's (the tokenizer is not on the path).
"""
from __future__ import annotations

from typing import Callable, Iterable, List, Sequence


def _valid_prefix(buf: bytes) -> int:
    """Length of the longest valid UTF-8 prefix (Rust's Utf8Error::valid_up_to)."""
    try:
        buf.decode("utf-8")
        return len(buf)
    except UnicodeDecodeError as e:
        return e.start


class ByteStream:
    """One sequence: push token bytes, get the text that became complete (main.rs:829-867)."""

    def __init__(self) -> None:
        self.pending = bytearray()

    def push(self, token_bytes: bytes) -> str:
        self.pending += token_bytes
        valid = _valid_prefix(bytes(self.pending))
        if valid == 0:
            return ""
        out = bytes(self.pending[:valid]).decode("utf-8")
        del self.pending[:valid]
        return out

    def flush(self) -> str:
        """The rest, lossily (main.rs:860-866, server.rs:213-215)."""
        out = bytes(self.pending).decode("utf-8", errors="replace")
        self.pending.clear()
        return out


class ByteStreams:
    """One ByteStream per row of a batched generation loop."""

    def __init__(self, rows: int, token_bytes: Callable[[int], bytes]) -> None:
        self.streams = [ByteStream() for _ in range(rows)]
        self.token_bytes = token_bytes

    def push(self, tokens: Sequence[int], active: Iterable[bool] | None = None) -> List[str]:
        """The text each row's new token completes ("" for rows not active)."""
        act = [True] * len(self.streams) if active is None else list(active)
        return [s.push(self.token_bytes(int(t))) if a else "" for s, t, a in zip(self.streams, tokens, act)]

    def flush(self) -> List[str]:
        return [s.flush() for s in self.streams]
