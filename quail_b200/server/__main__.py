"""Run Quail Server.

    python -m quail_b200.server --model qwen3-4b-fp8 --device b200 --data-dir ./quail-server [--port 50051]

Tables come from clients (DoPut) or from --parquet name=path arguments.
With QUAIL_SERVER_TOKEN set, clients must send it as a bearer token.
"""

from __future__ import annotations

import argparse


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(prog="quail-server")
    ap.add_argument("--model", required=True)
    ap.add_argument("--device", default="b200")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--weights", default=None)
    ap.add_argument("--tokenizer", default=None)
    ap.add_argument("--data-dir", required=True)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=50051)
    ap.add_argument("--parquet", action="append", default=[], help="name=path, registered at start")
    args = ap.parse_args(argv)
    import quail_b200 as quail
    from quail_b200.server.service import serve
    cfg = quail.EngineConfig(model=args.model, device=args.device, gpus=args.gpus, weights=args.weights,
                             tokenizer=args.tokenizer)
    session = quail.Session(config=cfg)
    for item in args.parquet:
        name, path = item.split("=", 1)
        session.register_parquet(name, path)
    print(f"quail-server on grpc://{args.host}:{args.port}, data in {args.data_dir}", flush=True)
    serve(session, args.data_dir, args.host, args.port)


if __name__ == "__main__":
    main()
