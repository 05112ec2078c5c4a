"""ORACLE (test infrastructure only): a pure-Python restatement of glypr's text front end.

Only ``tests/`` may import this module, as the checker of the library's tokenizer
(``glp_tokenizer_*``, ``glp_format_*``, ``glp_task_format``); the product never does.

What it restates (paths relative to crates/glypr-core/src of the reference):

* ``tokenizer.rs:77-138``  ``GlyprTokenizer::from_gguf_metadata``: vocabulary from
  ``tokenizer.ggml.tokens`` (token -> index, a later duplicate wins, as inserting into a hash
  map does), merges from ``tokenizer.ggml.merges`` (each string split on ' ', kept only when
  it has exactly two parts), a BPE model with byte fallback, fused unknowns and ``<unk>``,
  the normaliser Replace(' ' -> U+2581) and the pre-tokeniser Split(' ', MergedWithPrevious).
* The BPE model itself lives in the third-party crate ``tokenizers`` 0.22.2 (Cargo.lock:3151-3153,
  not vendored).  Its published algorithm, restated here: ``models/bpe/model.rs``
  ``BPE::build`` (merge map (left id, right id) -> (rank, id of the concatenation); an
  out-of-vocabulary part or concatenation is a build error; a later duplicate pair wins) and
  ``BPE::merge_word`` (one symbol per character; an unknown character falls back to its UTF-8
  bytes as ``<0xXX>`` tokens when all of them exist, else becomes ``<unk>``, consecutive unknowns
  fused into one; note that a byte fallback does not flush a pending unknown, which is emitted
  at the next known character or at the end of the word), and ``models/bpe/word.rs``
  ``Word::merge_all`` (a min-heap of candidate merges ordered by (rank, position); stale
  entries are skipped when the pair now at that position maps to a different new id).
  After the normaliser no ' ' is left, so the Split pre-tokeniser yields the whole text as one
  word.
* ``tokenizer.rs:162-177`` ``encode``: BPE ids, then BOS (2) prepended unless the first id is 2
  and EOS (1) appended unless the last id is 1 (the single-text path, ``lib.rs:968``).
* ``tokenizer.rs:454-566`` ``encode_modality_sequence`` for text parts: BOS, the BPE ids of
  prefix+text when non-empty, EOS (the batch and server path, ``lib.rs:833``,
  ``glypr-server/src/engine.rs:296-303``).
* ``tokenizer.rs:182-222`` ``encode_batch_padded_with_limit``: per-item limit check, right
  padding with 0 to the longest item.
* ``tokenizer.rs:13-64, 144-160`` ``default_prompts`` / ``format_query`` / ``format_document``
  and ``task.rs:21-73`` ``Task::prompt_prefix`` / ``format_text`` / ``from_name_and_title``.
  Rust's ``str::to_lowercase`` is Unicode's full default lowercase mapping with the Final_Sigma
  rule, which is what Python's ``str.lower`` implements too.

Pinned against ``tests/golden/tokenizer_golden.json``, made by ``tests/golden/make_tokenizer_golden.py``
with the Python binding of the same ``tokenizers`` crate version configured as
``from_gguf_metadata`` configures it, and against the reference's own known answers in
``task.rs:76-125``.
"""
from __future__ import annotations

import heapq
from typing import Dict, List, Optional, Sequence, Tuple

TOKEN_PAD, TOKEN_EOS, TOKEN_BOS = 0, 1, 2  # tokenizer.rs:588-590
DEFAULT_MAX_SEQ_LEN = 8192 + 128  # lib.rs:47

FORM_BARE, FORM_SINGLE, FORM_SEQUENCE = 0, 1, 2


class BuildError(Exception):
    pass


class EncodeError(Exception):
    pass


class BpeTokenizer:
    """The tokenizer ``from_gguf_metadata`` builds, from the two GGUF string arrays."""

    def __init__(self, tokens: Sequence[str], merges: Sequence[str], unk_token: str = "<unk>"):
        self.vocab: Dict[str, int] = {}
        for i, t in enumerate(tokens):  # tokenizer.rs:96-101: a later duplicate overwrites
            self.vocab[t] = i
        pairs: List[Tuple[str, str]] = []
        for m in merges:  # tokenizer.rs:103-111
            parts = m.split(" ")
            if len(parts) == 2:
                pairs.append((parts[0], parts[1]))
        # tokenizers models/bpe/model.rs BPE::build: rank = position in the list
        self.merges: Dict[Tuple[int, int], Tuple[int, int]] = {}
        for rank, (a, b) in enumerate(pairs):
            for part in (a, b, a + b):
                if part not in self.vocab:
                    raise BuildError(f"Token `{part}` out of vocabulary")
            self.merges[(self.vocab[a], self.vocab[b])] = (rank, self.vocab[a + b])
        self.unk_token = unk_token
        self.byte_ids = [self.vocab.get("<0x%02X>" % b) for b in range(256)]

    # -- models/bpe/model.rs merge_word ---------------------------------------------------
    def _word(self, w: str) -> List[List[int]]:
        """Symbols [id, prev, next, byte_len] of one word before merging."""
        syms: List[List[int]] = []

        def add(c: int, n: int) -> None:
            if syms:
                syms[-1][2] = len(syms)
                syms.append([c, len(syms) - 1, -1, n])
            else:
                syms.append([c, -1, -1, n])

        unk: Optional[List[int]] = None  # [id, byte_len] of the pending unknown
        for ch in w:
            blen = len(ch.encode("utf-8"))
            tid = self.vocab.get(ch)
            if tid is not None:
                if unk is not None:
                    add(unk[0], unk[1])
                    unk = None
                add(tid, blen)
                continue
            byte_ids = [self.byte_ids[b] for b in ch.encode("utf-8")]
            if all(b is not None for b in byte_ids):
                for b in byte_ids:  # the pending unknown stays pending
                    add(b, 1)
                continue
            if unk is not None:
                unk[1] += blen  # fuse_unk
            else:
                if self.unk_token not in self.vocab:
                    raise EncodeError(f"Unk token `{self.unk_token}` not found in the vocabulary")
                unk = [self.vocab[self.unk_token], blen]
        if unk is not None:
            add(unk[0], unk[1])
        return syms

    # -- models/bpe/word.rs merge_all -----------------------------------------------------
    def _merge_all(self, syms: List[List[int]]) -> List[int]:
        heap: List[Tuple[int, int, int]] = []  # (rank, pos, new_id): pops lowest rank, then pos
        for i in range(len(syms) - 1):
            m = self.merges.get((syms[i][0], syms[i + 1][0]))
            if m is not None:
                heap.append((m[0], i, m[1]))
        heapq.heapify(heap)
        while heap:
            rank, pos, new_id = heapq.heappop(heap)
            cur = syms[pos]
            if cur[3] == 0 or cur[2] == -1:
                continue
            nxt = cur[2]
            right = list(syms[nxt])
            m = self.merges.get((cur[0], right[0]))
            if m is None or m[1] != new_id:
                continue  # stale entry
            cur[0] = new_id
            cur[3] += right[3]
            cur[2] = right[2]
            syms[nxt][3] = 0
            if 0 <= right[2] < len(syms):
                syms[right[2]][1] = pos
            if cur[1] >= 0:
                m = self.merges.get((syms[cur[1]][0], cur[0]))
                if m is not None:
                    heapq.heappush(heap, (m[0], cur[1], m[1]))
            if 0 <= cur[2] < len(syms):
                m = self.merges.get((cur[0], syms[cur[2]][0]))
                if m is not None:
                    heapq.heappush(heap, (m[0], pos, m[1]))
        return [s[0] for s in syms if s[3] != 0]

    def bpe(self, text: str) -> List[int]:
        """``Tokenizer::encode(text, _)`` with no added tokens and no post-processor."""
        normalized = text.replace(" ", "▁")
        if not normalized:
            return []
        return self._merge_all(self._word(normalized))

    def encode(self, text: str, form: int = FORM_SINGLE) -> List[int]:
        ids = self.bpe(text)
        if form == FORM_SINGLE:  # tokenizer.rs:162-177
            if not ids or ids[0] != TOKEN_BOS:
                ids.insert(0, TOKEN_BOS)
            if ids[-1] != TOKEN_EOS:
                ids.append(TOKEN_EOS)
        elif form == FORM_SEQUENCE:  # tokenizer.rs:454-566, one text part
            ids = [TOKEN_BOS] + ids + [TOKEN_EOS]
        return ids

    def encode_batch_padded(self, texts: Sequence[str], limit: int, form: int = FORM_SINGLE):
        """tokenizer.rs:182-222: (ids [B, L] right-padded with 0, lengths)."""
        if not texts:
            raise EncodeError("Cannot encode an empty batch")
        rows = []
        for i, t in enumerate(texts):
            ids = self.encode(t, form)
            if len(ids) > limit:
                raise EncodeError(f"Batch item {i} sequence length ({len(ids)} tokens) exceeds maximum "
                                  f"context limit ({limit} tokens)")
            rows.append(ids)
        width = max(len(r) for r in rows)
        return [r + [TOKEN_PAD] * (width - len(r)) for r in rows], [len(r) for r in rows]


# -- prompts: tokenizer.rs:13-64, 144-160 ---------------------------------------------------
DEFAULT_PROMPTS = {
    "searchquery": "task: search result | query: ",
    "retrieval": "task: search result | query: ",
    "coderetrieval": "task: code retrieval | query: ",
    "questionanswering": "task: question answering | query: ",
    "factchecking": "task: fact checking | query: ",
    "sentencesimilarity": "task: sentence similarity | query: ",
    "sts": "task: sentence similarity | query: ",
    "summarization": "task: sentence similarity | query: ",
    "classification": "task: classification | query: ",
    "clustering": "task: clustering | query: ",
    "reranking": "task: search result | query: ",
    "bitextmining": "task: search result | query: ",
    "document": "title: none | text: ",
}


def _key(name: str) -> str:
    low = name.lower()
    for ch in "-_ ":
        low = low.replace(ch, "")
    return low


def format_query(query: str, task: str) -> str:
    prefix = DEFAULT_PROMPTS.get(_key(task))
    if prefix is None:
        prefix = f"task: {task.lower()} | query: "
    return prefix + query


def format_document(content: str, title: Optional[str]) -> str:
    return f"title: {title if title is not None else 'none'} | text: {content}"


# -- task.rs:21-73 ---------------------------------------------------------------------------
_TASK_NAMES = {
    "searchquery": "search", "retrieval": "search", "retrievalquery": "search", "query": "search",
    "document": "document", "retrievaldocument": "document",
    "coderetrieval": "code", "code": "code",
    "classification": "classification", "multilabelclassification": "classification",
    "clustering": "clustering",
    "questionanswering": "qa", "qa": "qa",
    "factchecking": "fact",
    "sentencesimilarity": "sts", "sts": "sts", "pairclassification": "sts", "summarization": "sts",
    "raw": "raw", "none": "raw",
}
_TASK_PREFIX = {
    "search": "task: search result | query: ",
    "code": "task: code retrieval | query: ",
    "classification": "task: classification | query: ",
    "clustering": "task: clustering | query: ",
    "qa": "task: question answering | query: ",
    "fact": "task: fact checking | query: ",
    "sts": "task: sentence similarity | query: ",
}


def task_prefix(name: Optional[str], title: Optional[str]) -> Optional[str]:
    """``Task::from_name_and_title(name, title).prompt_prefix()``; ``name`` None is Task::Raw."""
    if name is None:
        return None
    kind = _TASK_NAMES.get(_key(name))
    if kind == "raw":
        return None
    if kind == "document":
        return f"title: {title} | text: " if title is not None else "title: none | text: "
    if kind is not None:
        return _TASK_PREFIX[kind]
    if ":" in name or "|" in name:  # Task::Custom
        return name
    return f"task: {name} | query: "


def task_format(name: Optional[str], title: Optional[str], text: str) -> str:
    prefix = task_prefix(name, title)
    return text if prefix is None else prefix + text
