"""Public names of the plan types and prompt lowering.

- `PhysicalNode` / `PhysicalGraph`: the planner's node and plan
  (quail_b200.planner.plan.PlanNode / Plan): a node's kind (quail.scan,
  AiFilter, AiJoin, ...), its detail text, estimated rows and seconds, its
  inputs; the graph's nodes() and explain().
- `ExtensionNode`: a node an extension rule adds, marked with the
  extension's name.
- `ColumnRef`: a column of a relation, as prompts and providers name it.
- `lower_prompt`: a bound prompt's text pieces as the token ids a tokenizer
  gives them (the reference lowers prompts the same way: each piece
  tokenized on its own, quail/physical/lowering.py:174).
"""

from __future__ import annotations

from dataclasses import dataclass, field

from quail_b200.planner.plan import Plan as PhysicalGraph  # noqa: F401
from quail_b200.planner.plan import PlanNode as PhysicalNode


@dataclass
class ExtensionNode(PhysicalNode):
    """A plan node an extension contributed (its rule or runtime names it)."""

    extension: str = ""
    payload: dict = field(default_factory=dict)


@dataclass(frozen=True)
class ColumnRef:
    """One column of one relation: `relation.name`, or `name` when unqualified."""

    name: str
    relation: str | None = None

    def to_sql(self) -> str:
        return f"{self.relation}.{self.name}" if self.relation else self.name

    @classmethod
    def parse(cls, text: str) -> "ColumnRef":
        rel, dot, name = text.rpartition(".")
        return cls(name=name, relation=rel if dot else None)


@dataclass(frozen=True)
class LoweredPrompt:
    """A prompt as token ids: before the document, and after it (question + answer cue + turn end)."""

    preamble: tuple
    tail: tuple

    def around(self, document_ids) -> list[int]:
        return [*self.preamble, *document_ids, *self.tail]


def lower_prompt(prompt, tokenizer) -> LoweredPrompt:
    """`prompt` (from bind_prompt / bind_join_prompt) lowered with `tokenizer` (encode(text) -> ids)."""
    return LoweredPrompt(preamble=tuple(int(t) for t in tokenizer.encode(prompt.preamble)),
                         tail=tuple(int(t) for t in tokenizer.encode(prompt.tail)))
