"""ChatData (libr97host.so, host/chatdata.cpp; r97training_b200.data.ChatData) against the reference's own mask
test, tests/host/chatdata_mask.cpp: the expected ids are built here from the ChatML template as text
("<|im_start|>role\\ncontent<|im_end|>\\n") over the byte vocabulary, not from ChatData, so a moved mask boundary
fails -- an assistant message is scored on its content and its end-of-turn token, never on the role header or
the separator after the turn. The cases are that test's conversations (one turn, three turns, a system
message), its shortening boundaries, its three-conversation file, its skipped and malformed lines. CPU only."""
import json

import pytest

from r97training_b200.data import IM_END, IM_START, KEPT, SHORTENED, SKIPPED, ChatData, ChatDataError

ONE_TURN = [("user", "Hi"), ("assistant", "Hello!")]
THREE_TURNS = [("user", "Hi"), ("assistant", "Hello!"), ("user", "What is two plus two?"), ("assistant", "Four."),
               ("user", "Thanks"), ("assistant", "You are welcome!")]
WITH_SYSTEM = [("system", "You are terse."), ("user", "Hi"), ("assistant", "Hello!")]


def expected(messages):
    ids, score = [], []

    def text(t, s):
        for b in t.encode():
            ids.append(b)
            score.append(s)

    for role, content in messages:
        s = 1 if role == "assistant" else 0
        ids.append(IM_START)
        score.append(0)
        text(role, 0)
        text("\n", 0)
        text(content, s)
        ids.append(IM_END)
        score.append(s)
        text("\n", 0)
    return ids, score


def jsonl(*convs):
    return "\n".join(json.dumps({"messages": [{"role": r, "content": c} for r, c in conv]}) for conv in convs) + "\n"


def check(seq, want):
    assert seq.ids == want[0]
    assert seq.score == want[1]


def test_mask_one_turn():
    o, seq = ChatData().render(ONE_TURN)
    assert o == KEPT
    check(seq, expected(ONE_TURN))
    assert sum(seq.score) == 7  # the answer's six bytes and its end-of-turn token
    assert seq.score[0] == 0


def test_mask_three_turns():
    o, seq = ChatData().render(THREE_TURNS)
    assert o == KEPT
    check(seq, expected(THREE_TURNS))


def test_mask_with_system_message():
    o, seq = ChatData().render(WITH_SYSTEM)
    assert o == KEPT
    check(seq, expected(WITH_SYSTEM))
    assert seq.score[0] == 0 and seq.score[1] == 0


def test_shortens_trailing_turns_until_it_fits():
    cd = ChatData()
    one, two, full = expected(THREE_TURNS[:2]), expected(THREE_TURNS[:4]), expected(THREE_TURNS)
    assert len(full[0]) > len(two[0]) > len(one[0])
    o, seq = cd.render(THREE_TURNS, len(two[0]))  # exactly two turns fit: the third is dropped whole
    assert o == SHORTENED
    check(seq, two)
    o, seq = cd.render(THREE_TURNS, len(two[0]) - 1)
    assert o == SHORTENED
    check(seq, one)
    o, seq = cd.render(THREE_TURNS, len(one[0]))
    assert o == SHORTENED
    check(seq, one)
    o, seq = cd.render(THREE_TURNS, len(one[0]) - 1)  # the first exchange does not fit: skipped
    assert o == SKIPPED
    assert seq.ids == [] and seq.score == []


def test_trailing_user_turn_is_left_out_and_kept():
    o, seq = ChatData().render(ONE_TURN + [("user", "and then?")])
    assert o == KEPT  # rendered whole; only the message after the last assistant turn was left out
    check(seq, expected(ONE_TURN))


def test_reads_the_small_chat_file(tmp_path):
    path = tmp_path / "chat_small.jsonl"
    path.write_text(jsonl(ONE_TURN, THREE_TURNS, WITH_SYSTEM))
    cd = ChatData()
    batch = cd.read_file(str(path))
    st = cd.stats
    assert (st["conversations"], st["kept"], st["shortened"], st["skipped"]) == (3, 3, 0, 0)
    assert len(batch) == 3
    tokens = scored = 0
    for seq, conv in zip(batch, (ONE_TURN, THREE_TURNS, WITH_SYSTEM)):
        want = expected(conv)
        check(seq, want)
        tokens += len(want[0])
        scored += sum(want[1])
    assert st["tokens"] == tokens and st["scored"] == scored


def test_skips_a_conversation_with_no_assistant_turn():
    cd = ChatData()
    batch = cd.read('{"messages": [{"role": "user", "content": "Hi"}]}')
    assert cd.stats["conversations"] == 1 and cd.stats["skipped"] == 1 and cd.stats["kept"] == 0
    assert batch == []


def test_reports_a_malformed_line_and_its_number():
    cd = ChatData()
    text = ('{"messages": [{"role": "user", "content": "Hi"},{"role": "assistant", "content": "Hello!"}]}\n'
            '{"messages": 3}\n')
    with pytest.raises(ChatDataError) as e:
        cd.read(text)
    assert str(e.value).startswith("line 2:")
    assert "messages" in str(e.value)
    assert cd.stats["kept"] == 1  # the first line still counted, and its sequence appended
    assert cd._taken == 1


@pytest.mark.parametrize("line,why", [
    ("[1, 2]", "the line is not a JSON object"),
    ('{"messages": [1]}', "a message is not an object"),
    ('{"messages": [{"content": "x"}]}', 'a message has no string "role"'),
    ('{"messages": [{"role": "user", "content": 3}]}', 'the "user" message has no string "content"'),
    ('{"messages": [{"role": "user"', "the line is not a JSON object"),
])
def test_malformed_conversations(line, why):
    with pytest.raises(ChatDataError) as e:
        ChatData().line(line)
    assert str(e.value) == why


def test_json_escapes_and_unicode():
    """Escapes decode before rendering; content is scored byte for byte in UTF-8 (a surrogate pair too)."""
    content = 'tab\there "q" \\ é \U0001F600'
    line = json.dumps({"messages": [{"role": "user", "content": "x"}, {"role": "assistant", "content": content}]})
    o, seq = ChatData().line(line)
    assert o == KEPT
    check(seq, expected([("user", "x"), ("assistant", content)]))


def test_markers_in_content_are_parsed_as_control_tokens():
    """The renderer tokenises the rendered text with its specials parsed, as the reference's encode does
    (parse_special): an end-of-turn marker inside the answer ends the scored span there."""
    o, seq = ChatData().render([("user", "Hi"), ("assistant", "A<|im_end|>B")])
    assert o == KEPT
    assert seq.ids.count(IM_END) == 3
    scored = [i for i, s in zip(seq.ids, seq.score) if s]
    assert scored == [ord("A"), IM_END, ord("B"), IM_END]


def test_random_conversations_round_trip():
    """Seeded random conversations -- any code point (surrogate pairs included), escapes, extra keys and
    whitespace -- written by Python's json and read back: ids and mask as the template and the byte
    vocabulary give them."""
    import random
    rnd = random.Random(7)
    alphabet = list("ab /{}[]:,<|>") + ["\n", "\t", '"', "\\", "é", "中", "\U0001F600", "\u0007"]
    cd = ChatData()
    for _ in range(200):
        msgs = []
        for k in range(rnd.randint(1, 6)):
            role = rnd.choice(["system", "user", "assistant"]) if k else rnd.choice(["system", "user"])
            content = "".join(rnd.choice(alphabet) for _ in range(rnd.randint(0, 12)))
            msgs.append((role, content))
        doc = {"meta": {"n": rnd.random(), "tags": [1, None, True]},
               "messages": [{"role": r, "content": c, "extra": [1.5e-3]} for r, c in msgs]}
        line = json.dumps(doc, ensure_ascii=rnd.random() < 0.5, indent=rnd.choice([None, 1]))
        line = line.replace("\n", " ")
        o, seq = cd.line(line)
        last = max((i for i, (r, _) in enumerate(msgs) if r == "assistant"), default=-1)
        if last < 0:
            assert o == SKIPPED
            continue
        assert o == KEPT
        check(seq, expected(msgs[:last + 1]))
