"""Extracts the prompt-text fixtures of the reference's own tests for the EmbeddingGemma 2 texts.

    python tests/golden/make_prompt_golden.py /path/to/decision.js

Reads test/fixtures/prompts.json (the shared request states and questions) and test/fixtures/eg2-prompts.json
(the model's own renderings: render_state per state and workflow, render_question's question and option texts,
written by the reference's scripts/make-prompt-fixtures.py from the model's Python code) and writes
tests/golden/eg2_texts.json with the states, the questions and the expected texts. The token ids of those
fixtures are left out: they need the model's tokenizer.json, which is not in the reference's repository.
tests/test_prompts.py pins decision_js_b200.prompts against this file.
"""
import json
import os
import sys


def main(ref_root):
    fx = json.load(open(os.path.join(ref_root, "test", "fixtures", "prompts.json")))
    ex = json.load(open(os.path.join(ref_root, "test", "fixtures", "eg2-prompts.json")))
    out = {
        "source": "test/fixtures/prompts.json (states, questions), test/fixtures/eg2-prompts.json (texts)",
        "prompt": ex["prompt"],
        "states": fx["states"],
        "questions": fx["questions"],
        "state_texts": [{"state": c["state"], "workflow": c["workflow"], "text": c.get("text"),
                         "error": c.get("error")} for c in ex["states"]],
        "question_texts": [{"question": c["question"], "texts": c["texts"]} for c in ex["questions"]],
    }
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "eg2_texts.json")
    with open(path, "w") as f:
        json.dump(out, f, ensure_ascii=False, indent=0)
    print(path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_prompt_golden.py /path/to/decision.js")
    main(sys.argv[1])
