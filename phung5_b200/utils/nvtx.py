"""NVTX ranges for timeline profilers (PHX_NVTX=1): engine step phases and decoder layers.

Off by default (the push/pop calls cost host time on a launch-bound path); with PHX_NVTX=1 every engine
phase (setup, draft_catchup, draft_tree / graph_replay, select, verify, accept, commit_sync) and every
decoder layer of an eager forward is a named range.
"""
from __future__ import annotations

import os

import torch

ON = os.environ.get("PHX_NVTX") == "1" and torch.cuda.is_available()


def push(name: str) -> None:
    if ON:
        torch.cuda.nvtx.range_push(name)


def pop() -> None:
    if ON:
        torch.cuda.nvtx.range_pop()
