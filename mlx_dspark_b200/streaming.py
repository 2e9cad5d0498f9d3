"""Text streaming and stop strings of the decode loops (_Streamer, generate.py:294-362).

Every loop commits tokens a round at a time; after each round it hands the committed ids to
a TextStream, which turns the new ids into text, cuts the text at the first stop string
(and tells the loop to end), and passes newly settled text to the caller's on_text callback.
Text that could still turn out to be the start of a stop string (the last len(stop) - 1
characters) is held back until the next round or the end. A callback that raises
StopStreaming ends the decode at the next round boundary with a normal result. With neither
stop strings nor a callback the stream does nothing, so the loops' behaviour is unchanged.
"""
from __future__ import annotations


class StopStreaming(Exception):
    """Raised by an on_text callback to end a generation early (generate.py:229-233): the loop
    stops at the next round boundary and returns the partial result with
    finish_reason "stop"."""


class _WindowDecode:
    """Text of a growing id list that decodes a short window per new id instead of the whole
    list. The text of ids[start:mark] is already emitted; decoding ids[start:] and dropping
    that known text gives the new text. Starting the window one emitted piece back keeps the
    tokenizer's context for leading spaces. New text ending in U+FFFD (an incomplete
    multi-byte character) waits for the next id."""

    def __init__(self, tokenizer):
        self.tok = tokenizer
        self.ids: list[int] = []
        self.start = self.mark = 0
        self.pieces: list[str] = []

    def _take(self, force: bool) -> None:
        known = self.tok.decode(self.ids[self.start:self.mark])
        full = self.tok.decode(self.ids[self.start:])
        if len(full) > len(known) and (force or not full.endswith("\ufffd")):
            self.pieces.append(full[len(known):])
            self.start, self.mark = self.mark, len(self.ids)

    def add(self, token: int) -> None:
        self.ids.append(int(token))
        self._take(False)

    def finish(self) -> None:
        if self.mark < len(self.ids):
            self._take(True)

    @property
    def text(self) -> str:
        return "".join(self.pieces)


class _TokenizerDetok:
    """A tokenizer's own streaming detokenizer (mlx-lm's TokenizerWrapper.detokenizer:
    reset / add_token / finalize / text)."""

    def __init__(self, d):
        self.d = d
        if hasattr(d, "reset"):
            d.reset()

    def add(self, token: int) -> None:
        self.d.add_token(int(token))

    def finish(self) -> None:
        self.d.finalize()

    @property
    def text(self) -> str:
        return self.d.text


class TextStream:
    """Round-granular text of one decode: update(out_ids) after every round, flush() at the
    end; `stopped` turns true when a stop string appeared (or the callback asked to stop),
    and `text` is the output text cut before the earliest stop string."""

    def __init__(self, tokenizer, eos_ids, on_text=None, stop=None):
        self.stops = [s for s in (stop or []) if s]
        self.on_text = on_text
        self.active = on_text is not None or bool(self.stops)
        if self.active and (tokenizer is None or not hasattr(tokenizer, "decode")):
            raise ValueError("stop strings and on_text need a tokenizer with decode()")
        self.eos = set(eos_ids or ())
        # characters that may be the start of a stop string straddling two rounds
        self.hold = max((len(s) for s in self.stops), default=1) - 1
        self.detok = None
        if self.active:
            own = getattr(tokenizer, "detokenizer", None)
            self.detok = _TokenizerDetok(own) if own is not None else _WindowDecode(tokenizer)
        self.fed = 0          # ids of out_ids handed to the detokenizer
        self.scan_from = 0    # where the next stop-string search starts in the text
        self.emitted = 0      # characters passed to on_text
        self.text = ""
        self.stopped = False

    def update(self, out_ids: list[int]) -> None:
        if not self.active or self.stopped:
            return
        for t in out_ids[self.fed:]:
            if t not in self.eos:
                self.detok.add(t)
        self.fed = len(out_ids)
        self._settle(final=False)

    def flush(self) -> None:
        if not self.active or self.stopped:
            return
        self.detok.finish()
        self._settle(final=True)

    def _settle(self, final: bool) -> None:
        text = self.detok.text
        if self.stops:
            hits = [i for i in (text.find(s, self.scan_from) for s in self.stops) if i >= 0]
            if hits:
                text = text[:min(hits)]
                self.stopped = True
            else:
                self.scan_from = max(0, len(text) - self.hold)
        self.text = text
        if self.on_text is None:
            return
        upto = len(text) if (final or self.stopped) else max(self.emitted, len(text) - self.hold)
        if upto <= self.emitted:
            return
        try:
            self.on_text(text[self.emitted:upto])
        except StopStreaming:
            self.on_text = None   # nobody listens any more
            self.stopped = True
            return
        self.emitted = upto

    def final_text(self, tokenizer, out_ids: list[int], decode) -> str:
        """The result text: cut at the stop string when one was hit, else every non-eos id."""
        if self.stopped and self.active:
            return self.text
        return decode(tokenizer, [t for t in out_ids if t not in self.eos])
