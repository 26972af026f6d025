"""``avgen-b200`` command line (avgen/cli/main.py:79-88 API).

Exit codes: 0 success, 1 runtime error, 2 usage error, 3 configuration error,
130 interrupted.
"""
from __future__ import annotations

import argparse
import re
import sys
from collections.abc import Sequence

from avgen_b200.cli import checkpoint, data, evaluate, generate, info, plan, simulate, train
from avgen_b200.cli._common import EXIT_CONFIG, EXIT_ERROR, EXIT_INTERRUPT, EXIT_USAGE, fail, version

__all__ = ["build_parser", "main"]

_DESCRIPTION = """avgen-b200: train and sample video / audio-video diffusion transformers on B200.

  avgen-b200 plan --world-size 64 --seq-len 65536 --params 2e9 --depth 32 --width 2560
  avgen-b200 simulate --config run.yaml
  torchrun --nproc-per-node 8 -m avgen_b200.cli.main train --config run.yaml
  avgen-b200 generate --checkpoint runs/x/checkpoints/step_0000001000 --prompt "a red kite"
"""
_EPILOG = "exit codes: 0 ok, 1 runtime error, 2 usage error, 3 configuration error, 130 interrupted"


def build_parser() -> argparse.ArgumentParser:
    parser = argparse.ArgumentParser(prog="avgen-b200", description=_DESCRIPTION, epilog=_EPILOG,
                                     formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--version", action="store_true", help="print the version and exit")
    parser.add_argument("--traceback", action="store_true", help="show full tracebacks")
    sub = parser.add_subparsers(dest="command", metavar="COMMAND")
    for module in (train, generate, evaluate, simulate, plan, checkpoint, data, info):
        module.add_parser(sub)
    return parser


_OVERRIDE = re.compile(r"^[A-Za-z_][\w.\[\]-]*=")


def _overrides_last(argv: list[str]) -> list[str]:
    """Move ``key=value`` overrides behind the options so they may appear anywhere on the line
    (argparse only collects one contiguous run of positionals)."""
    moved, kept = [], []
    for i, tok in enumerate(argv):
        prev = argv[i - 1] if i else ""
        if _OVERRIDE.match(tok) and not prev.startswith("-"):
            moved.append(tok)
        else:
            kept.append(tok)
    return kept + moved


def main(argv: Sequence[str] | None = None) -> int:
    parser = build_parser()
    raw = list(argv) if argv is not None else sys.argv[1:]
    try:
        args = parser.parse_args(_overrides_last(raw))
    except SystemExit as exc:  # argparse: --help (0) or a usage error (2)
        return int(exc.code or 0)
    if args.version:
        sys.stdout.write(f"avgen-b200 {version()}\n")
        return 0
    handler = getattr(args, "handler", None)
    if handler is None:
        parser.print_help()
        return EXIT_USAGE
    try:
        return int(handler(args))
    except KeyboardInterrupt:
        sys.stderr.write("\navgen-b200: interrupted\n")
        return EXIT_INTERRUPT
    except Exception as exc:  # noqa: BLE001 - one line per failure unless --traceback
        if args.traceback:
            raise
        from avgen_b200.config.loader import ConfigError

        code = EXIT_CONFIG if isinstance(exc, ConfigError) else EXIT_ERROR
        return fail(f"{exc or type(exc).__name__}  (re-run with --traceback for frames)", code=code)


if __name__ == "__main__":
    raise SystemExit(main())
