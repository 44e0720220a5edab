"""Table providers: where a session's tables come from.

The reference's catalog (quail/catalog/providers.py) has the same shape: a
provider reports its columns and schema, a content identity (for caching),
statistics (row count), and scans record batches for a column projection.
`DocumentProvider.from_table` marks which column identifies a document.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass, field
from typing import Protocol

import pyarrow as pa


@dataclass(frozen=True)
class ScanRequest:
    columns: tuple | None = None
    limit: int | None = None
    batch_rows: int = 65_536


@dataclass(frozen=True)
class TableStatistics:
    num_rows: int | None = None


class TableProvider(Protocol):
    @property
    def columns(self) -> tuple[str, ...]: ...

    @property
    def schema(self) -> pa.Schema: ...

    def content_identity(self) -> str: ...

    def statistics(self) -> TableStatistics: ...

    def scan(self, request: ScanRequest) -> pa.RecordBatchReader: ...


def _check(schema: pa.Schema, request: ScanRequest) -> None:
    for c in request.columns or ():
        if c not in schema.names:
            raise KeyError(f"no column {c!r}; columns: {schema.names}")


@dataclass
class MemoryTableProvider:
    table: pa.Table

    @property
    def columns(self) -> tuple[str, ...]:
        return tuple(self.table.column_names)

    @property
    def schema(self) -> pa.Schema:
        return self.table.schema

    def content_identity(self) -> str:
        h = hashlib.sha256()
        for batch in self.table.to_batches():
            for col in batch.columns:
                for buf in col.buffers():
                    if buf is not None:
                        h.update(memoryview(buf))
        return h.hexdigest()[:16]

    def statistics(self) -> TableStatistics:
        return TableStatistics(self.table.num_rows)

    def scan(self, request: ScanRequest = ScanRequest()) -> pa.RecordBatchReader:
        _check(self.table.schema, request)
        t = self.table if request.columns is None else self.table.select(list(request.columns))
        if request.limit is not None:
            t = t.slice(0, request.limit)
        return pa.RecordBatchReader.from_batches(t.schema, t.to_batches(max_chunksize=request.batch_rows))


@dataclass
class ArrowDatasetProvider:
    """A parquet / json / csv file or directory read through pyarrow.dataset."""

    path: str
    format: str = "parquet"
    _dataset: object = field(default=None, repr=False)

    def _ds(self):
        if self._dataset is None:
            import pyarrow.dataset as ds
            self._dataset = ds.dataset(self.path, format=self.format)
        return self._dataset

    @property
    def columns(self) -> tuple[str, ...]:
        return tuple(self._ds().schema.names)

    @property
    def schema(self) -> pa.Schema:
        return self._ds().schema

    def content_identity(self) -> str:
        return hashlib.sha256(f"{self.format}:{self.path}".encode()).hexdigest()[:16]

    def statistics(self) -> TableStatistics:
        return TableStatistics(self._ds().count_rows())

    def scan(self, request: ScanRequest = ScanRequest()) -> pa.RecordBatchReader:
        _check(self.schema, request)
        scanner = self._ds().scanner(columns=list(request.columns) if request.columns else None,
                                     batch_size=request.batch_rows)
        reader = scanner.to_reader()
        if request.limit is None:
            return reader
        t = reader.read_all().slice(0, request.limit)
        return pa.RecordBatchReader.from_batches(t.schema, t.to_batches())


@dataclass
class DocumentProvider:
    """A table of documents with an identifying column."""

    inner: object
    id_col: str | None = None

    @classmethod
    def from_table(cls, table: pa.Table, id_col: str | None = None) -> "DocumentProvider":
        if id_col is not None and id_col not in table.column_names:
            raise KeyError(f"id column {id_col!r} not in {table.column_names}")
        return cls(MemoryTableProvider(table), id_col)

    @classmethod
    def from_parquet(cls, path: str, id_col: str | None = None) -> "DocumentProvider":
        return cls(ArrowDatasetProvider(path, "parquet"), id_col)

    @property
    def columns(self):
        return self.inner.columns

    @property
    def schema(self):
        return self.inner.schema

    def content_identity(self) -> str:
        return self.inner.content_identity()

    def statistics(self) -> TableStatistics:
        return self.inner.statistics()

    def scan(self, request: ScanRequest = ScanRequest()):
        return self.inner.scan(request)


def as_provider(obj) -> TableProvider:
    if isinstance(obj, pa.Table):
        return MemoryTableProvider(obj)
    if isinstance(obj, pa.RecordBatch):
        return MemoryTableProvider(pa.Table.from_batches([obj]))
    if hasattr(obj, "scan") and hasattr(obj, "schema"):
        return obj
    try:
        import pandas as pd
        if isinstance(obj, pd.DataFrame):
            return MemoryTableProvider(pa.Table.from_pandas(obj, preserve_index=False))
    except ImportError:
        pass
    raise TypeError(f"cannot register a {type(obj).__name__} as a table")
