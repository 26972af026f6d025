"""Shared teardown for the multi-GPU test workers (one process per rank)."""
from __future__ import annotations

import os
import sys
import traceback
from typing import NoReturn


def leave_on_failure() -> NoReturn:
    """Print the failure and end this rank at once.

    The other ranks may be blocked in a collective or a point-to-point receive that
    this rank will never join; meeting them in a barrier would hang every rank. The
    process exits instead, and the launcher (``torch.multiprocessing.spawn``) sees
    the non-zero exit code, stops the remaining ranks and fails the test.
    """
    traceback.print_exc()
    sys.stdout.flush()
    sys.stderr.flush()
    os._exit(1)
