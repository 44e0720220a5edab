"""Prompt text of each AI function call, in the model's chat format.

The prompt layout is an interface the answers depend on token for token, so
its strings are the same as the reference's
(crates/quail-planner/src/prompts.rs:16-31, the spec's turn_prefix /
turn_suffix in quail/specs/data/models/qwen3-4b-fp8.toml):

  turn_prefix + "DOCUMENT:\\n" + <document> +
  "\\n\\n" + "Evaluate TRUE or FALSE for the following question: " + <question> + "\\nANSWER:" +
  turn_suffix

A `PROMPT('<instruction> {0}', col)` template puts the document at {0}; the
text before the placeholder becomes the question asked after it (the
reference's "frame" move, prompts.rs:290-314).
"""

from __future__ import annotations

import re
from dataclasses import dataclass, field

SHARED_PRE = "DOCUMENT:\n"
JOIN_QUESTION_SEP = "\n\n"
TASK_INSTRUCTION = "Evaluate TRUE or FALSE for the following question: "
ANSWER_CUE = "\nANSWER:"
CLASSIFY_INSTRUCTION = "Answer with exactly one of the categories below for the following question: "
LETTERS_INSTRUCTION = "Answer with the letter of exactly one of the categories below for the following question: "
CATEGORIES_HEADER = "\n\nCategories:"
CHOICE_QUESTION = "Which option best fits the context?"
EXTRACT_QUESTION_LABEL = "\n\nQuestion: "
EXTRACT_INSTRUCTION = ("Copy the words that answer the question from the document. Copy them exactly. "
                       "Use the fewest words that answer it. If the document does not answer the question, "
                       "leave the phrase empty.")
EXTRACT_FORMAT = "Answer in this format:"
EXTRACT_PHRASE_FORMAT = "Phrase: <copied words>"
EXTRACT_PHRASE_CUE = "Phrase:"

QWEN3_TURN_PREFIX = "<|im_start|>system\nYou are an expert at text analysis<|im_end|>\n<|im_start|>user\n"
QWEN3_TURN_SUFFIX = "<|im_end|>\n<|im_start|>assistant\n<think>\n\n</think>\n\n"

# answer spellings read for AI.IF / AI.SCORE (the max over spellings is the side's logit)
TRUE_SPELLINGS = ("TRUE", " TRUE", "True", " True")
FALSE_SPELLINGS = ("FALSE", " FALSE", "False", " False")

_PLACEHOLDER = re.compile(r"\{(\d+)\}")


class PromptError(ValueError):
    pass


def placeholders(template: str) -> list[int]:
    return [int(m.group(1)) for m in _PLACEHOLDER.finditer(template)]


def check_placeholders(template: str, num_args: int) -> None:
    used = sorted(set(placeholders(template)))
    if num_args == 0:
        if used:
            raise PromptError(f"template uses placeholders {used} but no argument is given")
        return
    want = list(range(num_args))
    if used != want:
        raise PromptError(f"template placeholders {used} must be exactly {{0}}..{{{num_args - 1}}}")


@dataclass(frozen=True)
class Turn:
    prefix: str = QWEN3_TURN_PREFIX
    suffix: str = QWEN3_TURN_SUFFIX


@dataclass
class BoundPrompt:
    """A call's prompt split around the document.

    preamble: text before the document (turn prefix + "DOCUMENT:\\n"), shared
    by every row; tail: text after the document (question block + answer cue +
    turn suffix); question: the question text alone.
    """

    kind: str
    template: str
    preamble: str
    tail: str
    question: str
    labels: list = field(default_factory=list)
    descriptions: list = field(default_factory=list)

    def text(self, document: str) -> str:
        return self.preamble + document + self.tail


def split_frame(template: str) -> tuple[str, str]:
    """(question, rest after the document placeholder)."""
    i = template.find("{")
    if i < 0:
        return template.strip(), ""
    pre, tail = template[:i], template[i:]
    m = re.match(r"\{\d+\}", tail)
    if not m:
        raise PromptError("template text before the first placeholder must not contain a stray brace")
    question = pre.strip()
    rest = tail[m.end():]
    return question, rest


def bind_prompt(template: str, num_args: int = 1, turn: Turn = Turn()) -> BoundPrompt:
    """AI.IF / AI_FILTER prompt of a one-document template."""
    check_placeholders(template, num_args)
    if num_args > 1:
        raise PromptError("This filter must read a materialized document expression.")
    question, rest = split_frame(template)
    rest_q = rest.strip()
    if question and rest_q:
        question = f"{question}\n\n{rest_q}"
    elif rest_q:
        question = rest_q
    tail = JOIN_QUESTION_SEP + TASK_INSTRUCTION + question + ANSWER_CUE + turn.suffix
    return BoundPrompt(kind="filter", template=template, preamble=turn.prefix + SHARED_PRE, tail=tail,
                       question=question)


def bind_features_prompt(template: str, turn: Turn = Turn()) -> BoundPrompt:
    """AI.SAE_FEATURES: the user's prompt as written, in one user turn.

    The text after the document is required: the features are read at (or
    pooled up to) the prompt's tokens after the document
    (quail/backends/quail/executor/operators/sae_features.py:83-86).
    """
    check_placeholders(template, 1)
    i = template.find("{0}")
    head, rest = template[:i], template[i + 3:]
    if not rest.strip():
        raise PromptError("AI.SAE_FEATURES needs a question after the document")
    return BoundPrompt(kind="features", template=template, preamble=turn.prefix + head, tail=rest,
                       question=rest.strip())


def bind_score_prompt(template: str, num_args: int = 1, turn: Turn = Turn()) -> BoundPrompt:
    p = bind_prompt(template, num_args, turn)
    p.kind = "score"
    return p


def render_categories(labels: list[str], descriptions: list[str] | None = None) -> str:
    lines = []
    for i, label in enumerate(labels):
        d = descriptions[i] if descriptions and i < len(descriptions) and descriptions[i] else ""
        lines.append(f"- {label}: {d}" if d else f"- {label}")
    return CATEGORIES_HEADER + "\n" + "\n".join(lines)


def bind_classify_prompt(template: str | None, labels: list[str], descriptions: list[str] | None = None,
                         task_description: str = "", turn: Turn = Turn()) -> BoundPrompt:
    """AI.CLASSIFY prompt: the categories follow the question; the answer is a label."""
    if template:
        question, rest = split_frame(template)
        question = (question + ("\n\n" + rest.strip() if rest.strip() else "")).strip()
    else:
        question = ""
    if not question:
        question = task_description or CHOICE_QUESTION
    tail = (JOIN_QUESTION_SEP + CLASSIFY_INSTRUCTION + question + render_categories(labels, descriptions)
            + ANSWER_CUE + turn.suffix)
    return BoundPrompt(kind="classify", template=template or "", preamble=turn.prefix + SHARED_PRE, tail=tail,
                       question=question, labels=list(labels), descriptions=list(descriptions or []))


def bind_map_prompt(instruction: str, turn: Turn = Turn()) -> BoundPrompt:
    """AI.MAP: the document, then the instruction; the answer is free text."""
    tail = JOIN_QUESTION_SEP + instruction + turn.suffix
    return BoundPrompt(kind="map", template="{0}\n\n" + instruction, preamble=turn.prefix, tail=tail,
                       question=instruction)


def bind_extract_prompt(question: str, turn: Turn = Turn()) -> BoundPrompt:
    tail = (EXTRACT_QUESTION_LABEL + question + "\n\n" + EXTRACT_INSTRUCTION + "\n\n" + EXTRACT_FORMAT + "\n"
            + EXTRACT_PHRASE_FORMAT + turn.suffix + EXTRACT_PHRASE_CUE)
    return BoundPrompt(kind="extract", template="{0}", preamble=turn.prefix + SHARED_PRE, tail=tail,
                       question=question)


def bind_join_prompt(template: str, turn: Turn = Turn()) -> BoundPrompt:
    """Two-document AI.IF (a join): {0} and {1} become DOCUMENT 1 / DOCUMENT 2."""
    check_placeholders(template, 2)
    question = _PLACEHOLDER.sub("", template).strip()
    tail = JOIN_QUESTION_SEP + TASK_INSTRUCTION + question + ANSWER_CUE + turn.suffix
    return BoundPrompt(kind="join", template=template, preamble=turn.prefix, tail=tail, question=question)


# ---------------------------------------------------------------- model roles
#
# A model's role picks the prompt it reads (crates/quail-planner/src/prompts.rs:
# 144-178 for the decision2-noul layout; lowering.rs:448-465 for the Qwen3
# reranker's chat text). These strings are interfaces of the checkpoints, so
# they are the reference's, character for character.

DECISION2_DOCUMENT_LABEL = "Context:\n"
DECISION2_QUESTION_LABEL = "Task type: noul\nQuestion:\n"
DECISION2_CHOICE_LABEL = "Task type: choice\nQuestion:\n"
DECISION2_QUESTION_END = "\nOptions:"
DECISION2_CLOSING = ("\n\nSelect the single option best supported by the context and instructions."
                     "\nDecision:")
RERANKER_SYSTEM = ("You are an expert at text analysis. Judge whether the Document meets the requirements "
                   "based on the Query and the Instruct provided. Note that the answer can only be \"yes\" "
                   "or \"no\".")
RERANKER_INSTRUCTION = "Judge whether the document meets the requirements in the query."


# Base Labs' mammoth-1 / elephant-1 layout (crates/quail-planner/src/prompts.rs:131-140 and
# 191-201): the system turn and the document in a state block, then the question with lettered
# options and an answer line. A filter asks yes / no as options A and B. These strings are the
# checkpoints' interface, so they are the reference's, character for character.
MAMMOTH_DOCUMENT_LABEL = "<state>\n"
MAMMOTH_DOCUMENT_CLOSE = "\n</state>\n\n"
MAMMOTH_QUESTION_LABEL = "Question: "
MAMMOTH_OPTIONS_LABEL = "\n\nOptions:"
MAMMOTH_CLOSING = "\n\nAnswer with one letter: {letters}."
MAMMOTH_LABEL_CLOSING = "\n\nAnswer with one label: {letters}."
MAMMOTH_FILTER_END = ("\n\nOptions:\nA. yes: the statement is true / the answer is yes"
                      "\nB. no: the statement is false / the answer is no\n\nAnswer with one letter: A, B.")
MAMMOTH_EMPTY_QUESTION = "Which option applies to the state?"
MAX_LETTERS = 255          # the most options one coded prompt lists


# LiquidAI d1 layout (crates/quail-planner/src/prompts.rs:174-189): the document with no label,
# then "QUESTION:" blocks; the answer instructions, the option lines "<code> <text>", and the
# read slots are the checkpoint's interface, so they are the reference's
D1_QUESTION_SEPARATOR = "\n\n\n"
D1_QUESTION_LABEL = "QUESTION:\n"
D1_YES_NO_END = "\n\nReply with yes or no only."
D1_OPTION_END = "\n\nReply with the option code only."
D1_READ_END = "\n\nRead the text from the state, or nothing if it is absent."
D1_READ_SLOTS = "start:\nend:"


def code_candidates(n: int) -> list[str]:
    """The first n option codes: A to Z, then AA, AB, ... ZZ."""
    import string
    upper = list(string.ascii_uppercase)
    codes = upper + [a + b for a in upper for b in upper]
    return codes[:n]


@dataclass(frozen=True)
class PromptModel:
    """What the binder needs to know of a model: its role, prompt layout and chat turn."""

    role: str = "generative"
    layout: str = "ai-if"
    turn: Turn = Turn()
    name: str = ""


def prompt_model(cfg) -> PromptModel:
    """The prompt model of a decoder config: rerankers and decision models bring their own text."""
    role = getattr(cfg, "role", "generative")
    turn = Turn(prefix="", suffix="") if role in ("reranker", "decision") else Turn()
    if getattr(cfg, "turn_prefix", None) is not None:
        turn = Turn(prefix=cfg.turn_prefix, suffix=turn.suffix)
    if getattr(cfg, "turn_suffix", None) is not None:
        turn = Turn(prefix=turn.prefix, suffix=cfg.turn_suffix)
    return PromptModel(role=role, layout=getattr(cfg, "prompt_layout", "ai-if"), turn=turn,
                       name=getattr(cfg, "name", ""))


def decision2_option(key: str, description: str | None) -> str:
    """One option block: its fields as compact JSON with sorted keys."""
    import json
    body = json.dumps({"description": description, "key": key}, separators=(",", ":"), ensure_ascii=False,
                      sort_keys=True)
    return f"\n<option>\n{body}\n</option>"


@dataclass
class SegmentedPrompt(BoundPrompt):
    """A prompt whose tail is tokenized one segment at a time; `read` lists the
    segments whose last token the decision head reads (the last segment's last
    token, the prompt's last row, is always read)."""

    segments: list = field(default_factory=list)
    read: list = field(default_factory=list)


def bind_decision_prompt(template: str, kind: str, turn: Turn = Turn(prefix="", suffix="")) -> SegmentedPrompt:
    """AI.IF / AI.SCORE for a decision model: the question, then the options No and Yes."""
    base = bind_prompt(template, 1, turn)
    question = base.question
    segments = [JOIN_QUESTION_SEP + DECISION2_QUESTION_LABEL + question + DECISION2_QUESTION_END,
                decision2_option("false", "No"), decision2_option("true", "Yes"),
                DECISION2_CLOSING + turn.suffix]
    return SegmentedPrompt(kind=kind, template=template, preamble=turn.prefix + DECISION2_DOCUMENT_LABEL,
                           tail="".join(segments), question=question, segments=segments, read=[1, 2])


def bind_decision_choice_prompt(template: str | None, labels: list[str], descriptions: list[str] | None = None,
                                task_description: str = "",
                                turn: Turn = Turn(prefix="", suffix="")) -> SegmentedPrompt:
    """AI.CLASSIFY for a decision model: one option block per label, each read by the head."""
    if template:
        question, rest = split_frame(template)
        question = (question + ("\n\n" + rest.strip() if rest.strip() else "")).strip()
    else:
        question = ""
    if task_description:
        question = f"{question}\n{task_description}" if question else task_description
    question = question or CHOICE_QUESTION
    descriptions = list(descriptions or [])
    segments = [JOIN_QUESTION_SEP + DECISION2_CHOICE_LABEL + question + DECISION2_QUESTION_END]
    for i, label in enumerate(labels):
        d = descriptions[i] if i < len(descriptions) and descriptions[i] else None
        segments.append(decision2_option(str(label), d))
    segments.append(DECISION2_CLOSING + turn.suffix)
    return SegmentedPrompt(kind="classify", template=template or "", preamble=turn.prefix + DECISION2_DOCUMENT_LABEL,
                           tail="".join(segments), question=question, labels=list(labels),
                           descriptions=descriptions, segments=segments, read=list(range(1, len(labels) + 1)))


@dataclass
class LetteredPrompt(BoundPrompt):
    """A prompt answered by the LM head's logits of option letters at its last row (the
    slot_lm readout): option i is `letters[i]`; a filter's options are yes (A), then no (B)."""

    letters: list = field(default_factory=list)


def letter_candidates() -> list[str]:
    """Option letters for the letters rule: A to Z, a to z, then AA to ZZ."""
    import string
    upper = list(string.ascii_uppercase)
    return upper + list(string.ascii_lowercase) + [a + b for a in upper for b in upper]


def bind_letters_classify_prompt(template: str | None, labels: list[str], descriptions: list[str] | None = None,
                                 task_description: str = "", turn: Turn = Turn()) -> LetteredPrompt:
    """AI.CLASSIFY under the letters rule (a canvas model reads one row): the categories
    listed as "- <letter>: <label> (<description>)", answered by the logit of a letter."""
    if len(labels) > MAX_LETTERS:
        raise PromptError(f"a lettered prompt takes at most {MAX_LETTERS} options, got {len(labels)}")
    base = bind_classify_prompt(template, labels, descriptions, task_description, turn)
    letters = letter_candidates()[:len(labels)]
    lines = []
    for i, (letter, label) in enumerate(zip(letters, labels)):
        d = descriptions[i] if descriptions and i < len(descriptions) and descriptions[i] else ""
        lines.append(f"- {letter}: {label}" + (f" ({d})" if d else ""))
    tail = (JOIN_QUESTION_SEP + LETTERS_INSTRUCTION + base.question + CATEGORIES_HEADER + "\n" + "\n".join(lines)
            + ANSWER_CUE + turn.suffix)
    return LetteredPrompt(kind="classify", template=template or "", preamble=base.preamble, tail=tail,
                          question=base.question, labels=list(labels), descriptions=list(descriptions or []),
                          letters=letters)


def bind_mammoth_prompt(template: str, kind: str, turn: Turn = Turn(prefix="", suffix="")) -> LetteredPrompt:
    """AI.IF / AI.SCORE in the mammoth layout: the question, then options A (yes) and B (no)."""
    base = bind_prompt(template, 1, turn)
    question = base.question or MAMMOTH_EMPTY_QUESTION
    tail = MAMMOTH_QUESTION_LABEL + question + MAMMOTH_FILTER_END + turn.suffix
    return LetteredPrompt(kind=kind, template=template, preamble=turn.prefix + MAMMOTH_DOCUMENT_LABEL, tail=tail,
                          question=question, letters=["A", "B"])


def bind_mammoth_choice_prompt(template: str | None, labels: list[str], descriptions: list[str] | None = None,
                               task_description: str = "",
                               turn: Turn = Turn(prefix="", suffix="")) -> LetteredPrompt:
    """AI.CLASSIFY in the mammoth layout: one coded line per label, then the answer line
    (prompts.rs choice_segments: a two-letter code asks for "one label")."""
    if len(labels) > MAX_LETTERS:
        raise PromptError(f"a coded prompt takes at most {MAX_LETTERS} options, got {len(labels)}")
    if template:
        question, rest = split_frame(template)
        question = (question + ("\n\n" + rest.strip() if rest.strip() else "")).strip()
    else:
        question = ""
    if task_description:
        question = f"{question}\n{task_description}" if question else task_description
    question = question or MAMMOTH_EMPTY_QUESTION
    descriptions = list(descriptions or [])
    letters = code_candidates(len(labels))
    lines = "".join(f"\n{code}. {label}: {descriptions[i]}" if i < len(descriptions) and descriptions[i]
                    else f"\n{code}. {label}" for i, (code, label) in enumerate(zip(letters, labels)))
    closing = MAMMOTH_LABEL_CLOSING if any(len(c) > 1 for c in letters) else MAMMOTH_CLOSING
    tail = (MAMMOTH_QUESTION_LABEL + question + MAMMOTH_OPTIONS_LABEL + lines
            + closing.replace("{letters}", ", ".join(letters)) + turn.suffix)
    return LetteredPrompt(kind="classify", template=template or "", preamble=turn.prefix + MAMMOTH_DOCUMENT_LABEL,
                          tail=tail, question=question, labels=list(labels), descriptions=descriptions,
                          letters=letters)


def option_codes(labels: list[str]) -> list[str]:
    """A coded prompt's option codes: the labels themselves when every one is a single letter,
    else A, B, ... (prompts.rs option_codes)."""
    stripped = [str(x).strip() for x in labels]
    if stripped and all(len(x) == 1 and x.isalpha() for x in stripped):
        return stripped
    return code_candidates(len(labels))


def bind_d1_prompt(template: str, kind: str, turn: Turn = Turn(prefix="", suffix="")) -> LetteredPrompt:
    """AI.IF / AI.SCORE for a set-attention model: the question body after its header."""
    base = bind_prompt(template, 1, turn)
    return LetteredPrompt(kind=kind, template=template, preamble=turn.prefix,
                          tail=base.question + D1_YES_NO_END + turn.suffix, question=base.question)


def bind_d1_choice_prompt(template: str | None, labels: list[str], descriptions: list[str] | None = None,
                          task_description: str = "", turn: Turn = Turn(prefix="", suffix="")) -> LetteredPrompt:
    """AI.CLASSIFY for a set-attention model: the question, one "<code> <text>" line per option."""
    if template:
        question, rest = split_frame(template)
        question = (question + ("\n\n" + rest.strip() if rest.strip() else "")).strip()
    else:
        question = ""
    if task_description:
        question = f"{question}\n{task_description}" if question else task_description
    descriptions = list(descriptions or [])
    codes = option_codes(labels)
    lines = "\n".join(f"{code} {descriptions[i] if i < len(descriptions) and descriptions[i] else str(lab).replace('_', ' ')}"
                      for i, (code, lab) in enumerate(zip(codes, labels)))
    tail = question + "\n\nOptions:\n" + lines + D1_OPTION_END + turn.suffix
    return LetteredPrompt(kind="classify", template=template or "", preamble=turn.prefix, tail=tail,
                          question=question, labels=list(labels), descriptions=descriptions, letters=codes)


def bind_d1_read_prompt(question: str, turn: Turn = Turn(prefix="", suffix="")) -> BoundPrompt:
    """AI.EXTRACT for a set-attention model: a pointer read, answered at the two slot rows."""
    if not question.strip():
        raise PromptError("AI.EXTRACT needs a question with at least one word")
    return BoundPrompt(kind="extract", template="{0}", preamble=turn.prefix,
                       tail=question + D1_READ_END + turn.suffix + D1_READ_SLOTS, question=question)


def reranker_text(query: str, document: str) -> str:
    """The Qwen3 reranker's whole prompt for one (query, document) pair."""
    return ("<|im_start|>system\n" + RERANKER_SYSTEM + "<|im_end|>\n<|im_start|>user\n<Instruct>: "
            + RERANKER_INSTRUCTION + "\n<Query>: " + query + "\n<Document>: " + document
            + "<|im_end|>\n<|im_start|>assistant\n<think>\n\n</think>\n\n")


def bind_reranker_prompt(template: str) -> BoundPrompt:
    """AI.SCORE on a reranker: the query (the template without its document) goes before the document.

    The query is the template with a leading or trailing placeholder removed
    and any other occurrence read as "this document" (lowering.rs:420-446).
    """
    check_placeholders(template, 1)
    text = template.strip()
    if text.startswith("{0}"):
        text = text[3:].lstrip()
    if text.endswith("{0}"):
        text = text[:-3].rstrip()
    query = text.replace("{0}", "this document")
    before, after = reranker_text(query, "\x00").split("\x00")
    return BoundPrompt(kind="score", template=template, preamble=before, tail=after, question=query)
