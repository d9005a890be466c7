"""DeepSeek-V3.2 GR request layout and long-context experiment budgets.

Reference: ``models/deepseek_v32/request_format.py:1-16``.  A request is a chat
prefix (begin-of-sentence, instruction, user marker, "User history:"), the
user's history items, then the candidate items and the assistant ending.  The
tokenizer path is configurable (no fixed filesystem location is assumed).
"""

from __future__ import annotations

import os
from pathlib import Path

TOKENIZER_PATH = Path(os.environ.get("DEEPSEEK_TOKENIZER", "tokenizer.json"))
USER_LENGTHS = (4096, 16384, 65536, 262144, 1048576)
ITEM_LENGTHS = (64, 128, 256, 512, 1024, 2048, 4096)
MAX_INPUT_TOKENS = 1048576 + 4096
SPECIAL_TOKENS = ("<｜begin▁of▁sentence｜>", "<｜User｜>", "<｜Assistant｜>", "</think>")
ENDING = "<｜Assistant｜></think>"
BLOCK_CONTEXT = ""
TAIL_RESERVE_TOKENS = 2


def prefix(instruction: str) -> str:
    return f"<｜begin▁of▁sentence｜>{instruction}<｜User｜>User history:\n"
