"""Quail Server (Arrow Flight service + persistent query queue) and its client."""

from quail_b200.server.client import (  # noqa: F401
    QueryFailedError,
    QueryRun,
    QueryStatus,
    RemoteConnection,
    RemoteQuery,
    ServerClient,
)
