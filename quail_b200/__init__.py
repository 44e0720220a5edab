"""quail_b200: a B200-native engine for AI functions in SQL.

Public API (the same names as fsdatalab/quail's `quail` package):

    Session, EngineConfig, DocumentProvider, TableProvider, ScanRequest,
    Query, QueryResult, RefusalError, SHARED_PRE, bind_prompt,
    bind_join_prompt, speed_of_light_estimate
"""

from quail_b200.api.config import EngineConfig, Refusal, RefusalError  # noqa: F401
from quail_b200.api.prompts import SHARED_PRE, bind_join_prompt, bind_prompt  # noqa: F401
from quail_b200.api.session import Query, QueryResult, Session  # noqa: F401
from quail_b200.api.sol import SpeedOfLightEstimate, speed_of_light_estimate  # noqa: F401
from quail_b200.catalog import DocumentProvider, ScanRequest, TableProvider  # noqa: F401

__all__ = [
    "SHARED_PRE", "DocumentProvider", "EngineConfig", "Query", "QueryResult", "Refusal", "RefusalError",
    "ScanRequest", "Session", "SpeedOfLightEstimate", "TableProvider", "bind_join_prompt", "bind_prompt",
    "speed_of_light_estimate",
]
