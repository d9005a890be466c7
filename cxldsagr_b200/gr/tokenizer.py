"""Tokenizers for the GR workload.

``load_tokenizer(path)`` opens a HuggingFace ``tokenizer.json`` (e.g. the
DeepSeek-V3.2 tokenizer) with the ``tokenizers`` library.  Without one (no
network, no checkpoint), :func:`synthetic_tokenizer` builds a deterministic
word-level tokenizer over the generator's own vocabulary: words, single
digits, letters and punctuation each map to one id, and the DeepSeek chat
special tokens are added tokens.  Token counts are then additive across text
blocks, so exact per-request token budgets are reproducible offline, and all
ids stay below ``vocab_size`` of any model it is paired with (>= 512).
"""

from __future__ import annotations

import string
from pathlib import Path

from tokenizers import AddedToken, Tokenizer, models, pre_tokenizers

from ..models.deepseek_v32.request_format import SPECIAL_TOKENS

_WORDS = """
Recommend one item from the candidate pool based on the user history Output its index letter
User history profile Record Viewed Compared Saved Purchased Preference Candidate pool for visit
Details Looks good Quality is The design practical finish smooth size convenient Checked Catalog product
easy to clean comfortable use compact and lightweight suitable daily simple store designed travel
bag desk lamp water bottle running shoes wireless headphones coffee maker notebook storage box cotton
shirt face moisturizer blue green black white silver red
""".split()


def synthetic_tokenizer() -> Tokenizer:
    vocab = {"[UNK]": 0}
    for tok in list(dict.fromkeys(_WORDS)) + list(string.ascii_letters) + list(string.digits) + list(string.punctuation):
        vocab.setdefault(tok, len(vocab))
    tk = Tokenizer(models.WordLevel(vocab, unk_token="[UNK]"))
    tk.pre_tokenizer = pre_tokenizers.Sequence([
        pre_tokenizers.WhitespaceSplit(),
        pre_tokenizers.Punctuation(behavior="isolated"),
        pre_tokenizers.Digits(individual_digits=True),
    ])
    tk.add_special_tokens([AddedToken(t, special=True, normalized=False) for t in SPECIAL_TOKENS])
    return tk


def load_tokenizer(path: str | Path | None) -> Tokenizer:
    if path is None:
        return synthetic_tokenizer()
    p = Path(path)
    if p.is_dir():
        p = p / "tokenizer.json"
    return Tokenizer.from_file(str(p))
