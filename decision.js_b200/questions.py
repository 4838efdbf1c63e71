"""Questions and typed answers (src/questions.ts:1-45) and the host softmax (src/gpu.ts:294-297)."""
from __future__ import annotations

import json
import math


class QuestionError(ValueError):
    pass


def softmax(s):
    """softmax over a list of logits, in double precision on the host (src/gpu.ts:294-297)."""
    m = max(s)
    e = [math.exp(x - m) for x in s]
    z = sum(e)
    return [x / z for x in e]


def check_question(q: dict) -> dict:
    """Throws on a malformed question, with the reference's messages (src/questions.ts:19-29)."""
    if not isinstance(q, dict) or "type" not in q or "instructions" not in q:
        raise QuestionError("decision.js: a question is an object with `type`, `instructions` and, for choice and "
                            "score, `criteria`")
    t = q["type"]
    if t not in ("noul", "choice", "score"):
        raise QuestionError(f"decision.js: question type must be noul, choice or score, got {json.dumps(t, default=str)}")
    c = q.get("criteria")
    if t == "choice" and (not isinstance(c, dict) or len(c) < 2):
        raise QuestionError("decision.js: a choice needs criteria {name: description} with at least two options")
    if t == "score" and (not isinstance(c, list) or len(c) < 2 or len(c) > 10):
        raise QuestionError("decision.js: a score needs criteria: a list of 2 to 10 level descriptions, lowest first")
    if t == "noul" and c is not None and not isinstance(c, dict):
        raise QuestionError('decision.js: noul criteria are optional: {"true": "...", "false": "..."} (or "yes", "no")')
    return q


def answer(q: dict, probs, legend=str) -> dict:
    """A question's typed answer from its probabilities ([yes, no] for a noul, else option order)
    (src/questions.ts:32-44)."""
    if q["type"] == "noul":
        return {"type": "noul", "noul": probs[0]}
    best = 0
    for i, p in enumerate(probs):
        if p > probs[best]:
            best = i
    if q["type"] == "choice":
        names = list(q["criteria"].keys())
        return {"type": "choice", "choice": names[best], "confidence": probs[best],
                "probabilities": {n: probs[i] for i, n in enumerate(names)}}
    return {"type": "score", "score": sum(i * p for i, p in enumerate(probs)), "confidence": probs[best],
            "probabilities": {str(i): p for i, p in enumerate(probs)},
            "legend": {str(i): legend(c) for i, c in enumerate(q["criteria"])}}
