from quail_b200.catalog.providers import (  # noqa: F401
    ArrowDatasetProvider,
    DocumentProvider,
    MemoryTableProvider,
    ScanRequest,
    TableProvider,
    as_provider,
)
