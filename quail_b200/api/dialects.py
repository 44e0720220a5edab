"""SQL dialects a session accepts: Snowflake (the default) and BigQuery.

The parser reads one SQL grammar; a dialect only rewrites what the other
one spells differently before parsing:

- BigQuery quotes identifiers with backticks (`project.dataset.table`,
  `my col`): they become double-quoted identifiers, and a dotted path in one
  pair of backticks is its last part (the registered table's name);
- BigQuery's SAFE_CAST is CAST.

`SET datafusion.sql_parser.dialect = 'BigQuery'` (the reference's setting,
crates/quail-datafusion/src/lib.rs:106-120) switches a session's default.
"""

from __future__ import annotations

import re
from enum import Enum


class SQLDialect(str, Enum):
    SNOWFLAKE = "snowflake"
    BQ = "bq"

    @classmethod
    def of(cls, value) -> "SQLDialect":
        if isinstance(value, SQLDialect):
            return value
        v = str(value or "snowflake").lower()
        if v in ("bq", "bigquery"):
            return cls.BQ
        if v in ("snowflake", "generic", "default"):
            return cls.SNOWFLAKE
        raise ValueError(f"unknown SQL dialect {value!r}: use 'snowflake' or 'bq'")


_BACKTICK = re.compile(r"`([^`]*)`")


def _outside_strings(text: str, fn) -> str:
    """Apply fn to the parts of `text` outside single-quoted string literals."""
    out, i, n = [], 0, len(text)
    while i < n:
        j = text.find("'", i)
        if j < 0:
            out.append(fn(text[i:]))
            break
        out.append(fn(text[i:j]))
        k = j + 1
        while k < n:
            if text[k] == "'" and k + 1 < n and text[k + 1] == "'":
                k += 2
                continue
            if text[k] == "'":
                break
            k += 1
        out.append(text[j:k + 1])
        i = k + 1
    return "".join(out)


def to_parser_sql(text: str, dialect) -> str:
    """`text` in the parser's spelling."""
    if SQLDialect.of(dialect) is SQLDialect.SNOWFLAKE:
        return text

    def fix(part: str) -> str:
        part = _BACKTICK.sub(lambda m: '"' + m.group(1).split(".")[-1] + '"', part)
        return re.sub(r"\bSAFE_CAST\s*\(", "CAST(", part, flags=re.IGNORECASE)
    return _outside_strings(text, fix)
