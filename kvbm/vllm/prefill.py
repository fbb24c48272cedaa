"""``python -m kvbm.vllm.prefill``: vLLM's OpenAI-compatible API server with
the prefill-router attach.

Takes exactly the arguments of ``python -m vllm.entrypoints.openai.api_server``.
Before the server starts serving, the engine is handed to
:func:`kvbm_b200.hub.detect.try_wrap_engine`: when its connector
configuration names the ``prefill`` role, the process registers with the
hub's prefill router (``hub.url`` set) or serves the node's prefill plane
under its ``disagg.instance_id`` (no hub); otherwise it is plain vLLM. The
handler is kept alive for the life of the server.
"""

from __future__ import annotations

import logging

log = logging.getLogger(__name__)

_HANDLERS: list = []  # live prefill-router handlers (their hub registration ends when they are dropped)


def install_hook() -> None:
    """Wrap vLLM's ``build_and_serve`` so the engine is attached before the app serves."""
    from vllm.entrypoints.openai import api_server

    original = api_server.build_and_serve

    async def build_and_serve(engine_client, listen_address, sock, args, **kwargs):
        cfg = getattr(engine_client, "vllm_config", None)
        if cfg is not None:
            try:
                from kvbm_b200.hub.detect import try_wrap_engine

                handler = try_wrap_engine(cfg, engine_client)
                if handler is not None:
                    _HANDLERS.append(handler)
                    print(f"kvbm prefill server attached (instance {handler.instance_id})", flush=True)
            except Exception as e:  # noqa: BLE001 - the server still serves as plain vLLM
                log.warning("prefill-router attach failed: %s", e)
        return await original(engine_client, listen_address, sock, args, **kwargs)

    api_server.build_and_serve = build_and_serve


def main() -> None:
    logging.basicConfig(level=logging.INFO)
    install_hook()
    import uvloop
    from vllm.entrypoints.openai.api_server import cli_env_setup, make_arg_parser, run_server, validate_parsed_serve_args
    from vllm.utils.argparse_utils import FlexibleArgumentParser

    cli_env_setup()
    parser = make_arg_parser(FlexibleArgumentParser(description="vLLM API server with the kvbm prefill-router attach"))
    args = parser.parse_args()
    validate_parsed_serve_args(args)
    uvloop.run(run_server(args))


if __name__ == "__main__":
    main()
