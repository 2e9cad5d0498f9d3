"""Host-side text streaming of the decode loops (TextStream, mirroring _Streamer,
generate.py:294-362): incremental detokenization, stop strings that straddle rounds, the
held-back tail, StopStreaming from the callback, eos ids, and a tokenizer's own detokenizer.
Fake tokenizers, no GPU."""
import pytest

from mlx_dspark_b200.streaming import StopStreaming, TextStream


class CharTok:
    """id i -> one letter."""

    def decode(self, ids):
        return "".join(chr(97 + i % 26) for i in ids)


class ByteTok:
    """ids are UTF-8 bytes; incomplete characters decode to U+FFFD."""

    def decode(self, ids):
        return bytes(ids).decode("utf-8", errors="replace")


class SpaceTok:
    """Word pieces with a leading-space marker that decode() drops at the start of the text,
    as sentencepiece does."""

    vocab = ["▁the", "▁cat", "s", "▁sat", "▁on", "▁a", "▁mat", "."]

    def decode(self, ids):
        return "".join(self.vocab[i] for i in ids).replace("▁", " ").lstrip(" ")


def _run(stream, ids, per_round):
    out = []
    for i in range(0, len(ids), per_round):
        if stream.stopped:
            break
        out.extend(ids[i:i + per_round])
        stream.update(out)
    stream.flush()
    return out


def test_inactive_stream_needs_nothing():
    st = TextStream(None, set())
    st.update([1, 2, 3])
    st.flush()
    assert not st.stopped and st.final_text(None, [1, 2], lambda t, ids: "x") == "x"
    with pytest.raises(ValueError):
        TextStream(None, set(), stop=["a"])


def test_stop_string_straddling_rounds_and_held_tail():
    got = []
    st = TextStream(CharTok(), set(), on_text=got.append, stop=["cde"])
    ids = list(range(10))                     # "abcdefghij"
    out = _run(st, ids, 3)                    # rounds "abc", "def": "cde" straddles them
    assert st.stopped and st.text == "ab"
    assert "".join(got) == "ab"
    assert out == list(range(6))              # the loop stops at the round boundary
    assert st.final_text(CharTok(), out, None) == "ab"


def test_earliest_of_several_stop_strings():
    st = TextStream(CharTok(), set(), stop=["ghi", "def", "zz"])
    _run(st, list(range(10)), 4)
    assert st.stopped and st.text == "abc"


def test_emission_holds_back_a_possible_stop_prefix():
    calls = []
    st = TextStream(CharTok(), set(), on_text=calls.append, stop=["xyz"])
    out = []
    for i in range(0, 8, 2):
        out.extend([i, i + 1])
        st.update(out)
        # everything but the last 2 characters has been handed out
        assert "".join(calls) == CharTok().decode(out)[:len(out) - 2]
    st.flush()
    assert "".join(calls) == "abcdefgh" and not st.stopped


def test_stop_streaming_from_callback():
    calls = []

    def cb(s):
        calls.append(s)
        if len(calls) == 2:
            raise StopStreaming()

    st = TextStream(CharTok(), set(), on_text=cb)
    out = _run(st, list(range(12)), 2)
    assert st.stopped and len(calls) == 2 and out == list(range(4))


def test_multibyte_characters_wait_for_their_last_byte():
    text = "héllo wörld ☃!"
    ids = list(text.encode("utf-8"))
    got = []
    st = TextStream(ByteTok(), set(), on_text=got.append)
    _run(st, ids, 1)
    assert "".join(got) == text and "�" not in "".join(got)


def test_leading_spaces_survive_the_window():
    ids = [0, 1, 2, 3, 4, 5, 6, 7]
    got = []
    st = TextStream(SpaceTok(), set(), on_text=got.append)
    _run(st, ids, 3)
    assert "".join(got) == SpaceTok().decode(ids) == "the cats sat on a mat."


def test_eos_ids_are_not_text():
    st = TextStream(CharTok(), {25}, stop=["q"])
    _run(st, [0, 25, 1, 25, 2], 2)
    assert st.text == "abc"
    assert st.final_text(CharTok(), [0, 25, 1], lambda t, ids: t.decode(ids)) == "ab"


def test_tokenizer_own_detokenizer_is_used():
    class Detok:
        def __init__(self):
            self.ids, self.resets, self.final = [], 0, False

        def reset(self):
            self.ids, self.resets = [], self.resets + 1

        def add_token(self, t):
            self.ids.append(t)

        def finalize(self):
            self.final = True

        @property
        def text(self):
            return "".join(str(i) for i in self.ids)

    class Tok:
        detokenizer = Detok()

        def decode(self, ids):
            raise AssertionError("the window decoder should not run")

    st = TextStream(Tok(), set(), stop=["34"])
    _run(st, [1, 2, 3, 4, 5], 2)
    assert st.stopped and st.text == "12" and Tok.detokenizer.resets == 1
