"""The host pipeline in front of the pass (decision_js_b200.prompts): the EmbeddingGemma 2 texts pinned against the
reference's own prompt fixtures (tests/golden/eg2_texts.json, extracted by tests/golden/make_prompt_golden.py from
test/fixtures/eg2-prompts.json and prompts.json), Python's renderings, the tokenizer interface and the d1-3B prompt's
structure (src/d1-3b-prompt.ts)."""
import json
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
G = json.load(open(os.path.join(HERE, "golden", "eg2_texts.json")))


def test_eg2_state_texts_match_the_reference_fixtures(pkg):
    """renderState on every fixture state and workflow (src/eg2-prompt.ts:14-28); the states the model itself
    refuses (a string that only starts like JSON) render as plain text, as the reference's test allows."""
    from decision_js_b200 import prompts
    assert len(G["state_texts"]) == 14
    for c in G["state_texts"]:
        text = prompts.render_state(G["states"][c["state"]], c["workflow"])
        if c["error"]:
            assert text.startswith("workflow: ")
        else:
            assert text == c["text"], (c["state"], c["workflow"])


def test_eg2_question_texts_match_the_reference_fixtures(pkg):
    """renderQuestion on every fixture question: the question text and each option's, in option order
    (src/eg2-prompt.ts:32-40)."""
    from decision_js_b200 import prompts
    assert len(G["question_texts"]) == 9
    for c in G["question_texts"]:
        q, opts = prompts.render_question(G["questions"][c["question"]], "q")
        assert [q] + opts == c["texts"], c["question"]


def test_python_renderings(pkg):
    """str() / json.dumps / repr as prompt.py writes them (src/py.ts), with JavaScript's one number type."""
    from decision_js_b200 import prompts as P
    assert P.py_str(None) == "None" and P.py_str(True) == "True" and P.py_str(3) == "3"
    assert P.py_str(1.0) == "1" and P.py_str(1234.5) == "1234.5" and P.py_str(1e-5) == "1e-05"
    assert P.py_str(1.5e16) == "1.5e+16" and P.py_str(float("nan")) == "nan" and P.py_str(float("-inf")) == "-inf"
    assert P.py_str(["a", 1, {"b": [2, 3]}]) == "['a', 1, {'b': [2, 3]}]"
    assert P.py_str({"it's": 'say "hi"'}) == '{"it\'s": \'say "hi"\'}'
    assert P.py_str(["x\ny\t\x01"]) == "['x\\ny\\t\\x01']"
    assert P.py_dumps({"a": [1, 2.5, None, True], "é": "ü"}) == '{"a": [1, 2.5, null, true], "é": "ü"}'
    assert P.py_dumps({"a": {"b": []}}, 2) == '{\n  "a": {\n    "b": []\n  }\n}'
    assert P.py_dumps(float("inf")) == "Infinity"
    assert [P.py_truthy(v) for v in (None, 0, 0.0, "", [], {}, False, 1, "x", [0], {"a": 1})] == \
        [False] * 7 + [True] * 4
    assert P.criterion("text") == "text" and P.criterion({"a": 1}) == '{"a": 1}'


@pytest.fixture(scope="module")
def tok_dir(tmp_path_factory, pkg):
    from decision_js_b200 import prompts, synth
    d = str(tmp_path_factory.mktemp("tok"))
    texts = [c["text"] for c in G["state_texts"] if c["text"]] + [t for c in G["question_texts"] for t in c["texts"]]
    texts += [G["prompt"], "Options Reply with the option code only yes or no single digit QUESTION user assistant"]
    texts += [prompts.D13BPrompt(None).question_block(q) if q["type"] != "choice" else "" for q in G["questions"]]
    synth.write_tokenizer(d, texts, 8192)
    return d


def test_tokenizer_and_eg2_tokenize(pkg, tok_dir):
    """<bos> prompt + text <eos>, truncated to max_len tokens (src/eg2-prompt.ts:43-46); special tokens written in
    the text still match (src/tokenizer.ts:20-23)."""
    from decision_js_b200 import prompts
    tok = prompts.TextTokenizer.load(tok_dir)
    bos, eos = tok.id("<bos>"), tok.id("<eos>")
    assert tok.special("bos_token") == "<bos>" and tok.bos == "<bos>"
    ids = prompts.tokenize(tok, "hello <eos> world", G["prompt"])
    assert ids[0] == bos and ids[-1] == eos and eos in ids[1:-1]
    assert ids[1:-1] == tok.encode(G["prompt"] + "hello <eos> world")
    short = prompts.tokenize(tok, "a b c d e f g", G["prompt"], max_len=6)
    assert len(short) == 6 and short[0] == bos and short[-1] == eos
    with pytest.raises(ValueError):
        tok.special("mask_token")


def test_d13b_prompt_structure(pkg, tok_dir):
    """The d1-3B trunk ends at QUESTION:, a branch ends at the assistant header, and each option's readout group
    holds single-token forms (src/d1-3b-prompt.ts:68-122)."""
    from decision_js_b200 import prompts
    tok = prompts.TextTokenizer.load(tok_dir)
    p = prompts.D13BPrompt(tok)
    state = G["states"][1]
    pre = p.prefix_text(state)
    assert pre.startswith("<bos><|im_start|>user\n{\n  \"subject\"") and pre.endswith("\n\n\nQUESTION:\n")
    assert p.prefix_text(None) == "<bos><|im_start|>user\n"
    assert p.prefix_text("plain") == "<bos><|im_start|>user\nplain\n\n\nQUESTION:\n"
    for q in G["questions"]:
        suf = p.suffix_text(q)
        assert suf.startswith(str(q["instructions"])) and suf.endswith("<|im_end|>\n<|im_start|>assistant\n")
        groups = p.readout_ids(q)
        n = 2 if q["type"] == "noul" else len(q["criteria"])
        assert len(groups) == n and all(len(g) >= 1 for g in groups)
        assert len({g[0] for g in groups}) == n  # distinct codes
    choice = next(q for q in G["questions"] if q["type"] == "choice")
    block = p.question_block(choice)
    assert "\n\nOptions:\nA " in block and block.endswith("\n\nReply with the option code only.")
    noul = {"type": "noul", "instructions": "Spam?", "criteria": {"true": "junk", "false": "fine"}}
    assert p.question_block(noul) == "Spam?\nYes: junk\nNo: fine\n\nReply with yes or no only."
    score = {"type": "score", "instructions": "Level?", "criteria": ["low", "high"]}
    assert p.question_block(score) == "Level?\n\n0 low\n1 high\n\nReply with a single digit 0-1 only."
    assert prompts.option_codes(["a", "b"]) == ["a", "b"] and prompts.option_codes(["ab", "c"]) == ["A", "B"]
    assert prompts.option_codes([str(i) for i in range(30)])[:2] == ["00", "01"]
    assert p.trunk(state) == tok.encode(pre) and np.all(np.array(p.branch(choice)) >= 0)
