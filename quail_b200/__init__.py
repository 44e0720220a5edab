"""quail_b200: a B200-native engine for AI functions in SQL.

Public API (the same names as fsdatalab/quail's `quail` package):

    Session, EngineConfig, DocumentProvider, TableProvider, ScanRequest,
    Query, QueryResult, RefusalError, SHARED_PRE, bind_prompt,
    bind_join_prompt, lower_prompt, speed_of_light_estimate,
    SpeedOfLightEstimate, SQLDialect, ColumnRef, ExtensionRegistry,
    PhysicalGraph, PhysicalNode, ExtensionNode, QueryRun, QueryStatus,
    QueryFailedError
"""

from quail_b200.api.config import EngineConfig, Refusal, RefusalError  # noqa: F401
from quail_b200.api.prompts import SHARED_PRE, bind_join_prompt, bind_prompt  # noqa: F401
from quail_b200.api.session import Query, QueryResult, Session  # noqa: F401
from quail_b200.api.sol import SpeedOfLightEstimate, speed_of_light_estimate  # noqa: F401
from quail_b200.catalog import DocumentProvider, ScanRequest, TableProvider  # noqa: F401
from quail_b200.api.dialects import SQLDialect  # noqa: F401
from quail_b200.api.physical import ColumnRef, ExtensionNode, PhysicalGraph, PhysicalNode, lower_prompt  # noqa: F401
from quail_b200.extensions import ExtensionRegistry  # noqa: F401
from quail_b200.server.client import QueryFailedError, QueryRun, QueryStatus  # noqa: F401

__all__ = [
    "SHARED_PRE", "ColumnRef", "DocumentProvider", "EngineConfig", "ExtensionNode", "ExtensionRegistry",
    "PhysicalGraph", "PhysicalNode", "Query", "QueryFailedError", "QueryResult", "QueryRun", "QueryStatus",
    "Refusal", "RefusalError", "SQLDialect", "ScanRequest", "Session", "SpeedOfLightEstimate", "TableProvider",
    "bind_join_prompt", "bind_prompt", "lower_prompt", "speed_of_light_estimate",
]
