"""Incremental UTF-8 output (lrs.stream), after rust-llama's ByteStream (main.rs:829-867) and
the server's generation core (server.rs:186-215): complete UTF-8 is emitted as soon as a token
completes it, incomplete sequences wait, invalid bytes wait until the final lossy flush."""
from lrs.stream import ByteStream, ByteStreams


def test_multibyte_character_split_across_tokens():
    s = ByteStream()
    euro = "€".encode()  # e2 82 ac
    assert s.push(b"a") == "a"
    assert s.push(euro[:1]) == ""
    assert s.push(euro[1:2]) == ""
    assert s.push(euro[2:] + b"b") == "€b"
    assert s.flush() == ""


def test_complete_prefix_emitted_and_tail_kept():
    s = ByteStream()
    word = "héllo👍".encode()
    assert s.push(word[:-2]) == "héllo"  # the emoji's last two bytes are missing
    assert bytes(s.pending) == word[-4:-2]
    assert s.push(word[-2:]) == "👍"


def test_invalid_bytes_wait_for_the_lossy_flush():
    # valid_up_to stops at an invalid byte: nothing after it is emitted until the end
    s = ByteStream()
    assert s.push(b"ok\xff") == "ok"
    assert s.push(b"more") == ""
    assert s.flush() == "�more"
    assert s.flush() == ""


def test_lossy_flush_of_an_incomplete_sequence():
    s = ByteStream()
    assert s.push("ü".encode()[:1]) == ""
    assert s.flush() == "�"


def test_rows_of_a_batch_are_independent():
    table = {0: b"x", 1: "ß".encode()[:1], 2: "ß".encode()[1:], 3: b"\n"}
    st = ByteStreams(3, lambda t: table[t])
    assert st.push([0, 1, 3]) == ["x", "", "\n"]
    assert st.push([1, 2, 0], active=[True, True, False]) == ["", "ß", ""]
    assert st.push([3, 3, 3]) == ["", "\n", "\n"]  # row 0: 0xc3 then a newline, invalid: it waits
    assert st.flush() == ["�\n", "", ""]
