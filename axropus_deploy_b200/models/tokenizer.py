"""BPE tokenizer read from a Hugging Face ``tokenizer.json``.

Covers the two families the served models use:

* byte-level BPE (Llama-3): a regex split of the text, each piece mapped byte by byte
  to printable characters (the GPT-2 byte table), then merged by rank; with
  ``ignore_merges`` a piece that is itself a vocabulary entry is taken whole;
* Metaspace / SentencePiece-style BPE (Llama-2, Mistral, Mixtral): spaces replaced by
  ``▁`` (and one prepended), merged by rank, characters outside the vocabulary spelled
  as ``<0xNN>`` byte tokens (``byte_fallback``).

Special tokens (``added_tokens``) are cut out of the text before anything else and map
to their ids; ``encode(..., add_special_tokens=True)`` applies the post-processor's
single-sequence template (e.g. a leading ``<|begin_of_text|>``). ``decode`` inverts the
byte table or the ``▁`` / byte-token spelling. The algorithm follows the published BPE
method (Sennrich, Haddow & Birch 2016: repeatedly merge the adjacent pair of lowest
rank) and the tokenizer.json format; tests compare it with the ``tokenizers`` library.
"""
from __future__ import annotations

import json
import unicodedata
from functools import lru_cache
from typing import Dict, List, Optional, Sequence, Tuple

import regex

# GPT-2 style split, used by a ByteLevel pre-tokenizer with use_regex
_GPT2_SPLIT = r"""'s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+"""


def _byte_table() -> Dict[int, str]:
    """Byte -> printable character: printable Latin-1 bytes map to themselves, the other
    bytes to code points from 256 upward, in byte order."""
    keep = list(range(ord("!"), ord("~") + 1)) + list(range(ord("¡"), ord("¬") + 1)) + \
        list(range(ord("®"), ord("ÿ") + 1))
    table, extra = {}, 0
    for b in range(256):
        if b in keep:
            table[b] = chr(b)
        else:
            table[b] = chr(256 + extra)
            extra += 1
    return table


_B2U = _byte_table()
_U2B = {u: b for b, u in _B2U.items()}


class Tokenizer:
    def __init__(self, spec: dict):
        m = spec["model"]
        if m.get("type", "BPE") != "BPE":
            raise ValueError(f"tokenizer model {m.get('type')!r} is not supported (BPE only)")
        self.vocab: Dict[str, int] = dict(m["vocab"])
        merges = m.get("merges", [])
        pairs = [tuple(x.split(" ", 1)) if isinstance(x, str) else tuple(x) for x in merges]
        self.ranks: Dict[Tuple[str, str], int] = {p: i for i, p in enumerate(pairs)}
        self.byte_fallback = bool(m.get("byte_fallback", False))
        self.ignore_merges = bool(m.get("ignore_merges", False))
        self.unk = m.get("unk_token")
        self.fuse_unk = bool(m.get("fuse_unk", False))
        self.added: Dict[str, int] = {}
        self.special_ids = set()
        for t in spec.get("added_tokens", []) or []:
            self.added[t["content"]] = int(t["id"])
            if t.get("special", False):
                self.special_ids.add(int(t["id"]))
        self.id_to_token: Dict[int, str] = {i: t for t, i in self.vocab.items()}
        self.id_to_token.update({i: t for t, i in self.added.items()})
        self._added_re = regex.compile("|".join(regex.escape(t) for t in sorted(self.added, key=len, reverse=True))) \
            if self.added else None
        self.normalizer = spec.get("normalizer")
        self.pre = spec.get("pre_tokenizer")
        self.post = spec.get("post_processor")
        self.decoder = spec.get("decoder")
        self.byte_level = self._has(self.pre, "ByteLevel") or self._has(self.decoder, "ByteLevel")
        self._cache = lru_cache(maxsize=65536)(self._bpe)

    @classmethod
    def from_file(cls, path: str) -> "Tokenizer":
        with open(path, encoding="utf-8") as f:
            return cls(json.load(f))

    @staticmethod
    def _has(node, kind: str) -> bool:
        if not node:
            return False
        if node.get("type") == kind:
            return True
        return any(Tokenizer._has(x, kind) for x in node.get("pretokenizers", []) + node.get("decoders", []) +
                   node.get("normalizers", []))

    @property
    def vocab_size(self) -> int:
        return max(self.id_to_token) + 1 if self.id_to_token else 0

    # ------------------------------------------------------------------ normalize / split
    def _normalize(self, s: str, node=None) -> str:
        node = self.normalizer if node is None else node
        if not node:
            return s
        t = node.get("type")
        if t == "Sequence":
            for n in node["normalizers"]:
                s = self._normalize(s, n)
            return s
        if t == "Prepend":
            return node["prepend"] + s if s else s
        if t == "Replace":
            pat = node["pattern"]
            return s.replace(pat["String"], node["content"]) if "String" in pat else \
                regex.sub(pat["Regex"], node["content"], s)
        if t in ("NFC", "NFD", "NFKC", "NFKD"):
            return unicodedata.normalize(t, s)
        if t == "Lowercase":
            return s.lower()
        raise ValueError(f"normalizer {t!r} is not supported")

    def _split(self, pieces: List[str], node) -> List[str]:
        if not node:
            return pieces
        t = node.get("type")
        if t == "Sequence":
            for n in node["pretokenizers"]:
                pieces = self._split(pieces, n)
            return pieces
        out: List[str] = []
        if t == "Split":
            pat = node["pattern"]
            rx = regex.compile(pat["Regex"] if "Regex" in pat else regex.escape(pat["String"]))
            behavior = node.get("behavior", "Isolated")
            for p in pieces:
                pos = 0
                for mt in rx.finditer(p):
                    if mt.start() > pos:
                        out.append(p[pos:mt.start()])
                    if behavior != "Removed" and mt.end() > mt.start():
                        out.append(mt.group())
                    pos = mt.end()
                if pos < len(p):
                    out.append(p[pos:])
            return [x for x in out if x]
        if t == "ByteLevel":
            for p in pieces:
                if node.get("add_prefix_space", False) and not p.startswith(" "):
                    p = " " + p
                parts = regex.findall(_GPT2_SPLIT, p) if node.get("use_regex", True) else [p]
                out += ["".join(_B2U[b] for b in x.encode("utf-8")) for x in parts]
            return out
        if t == "Metaspace":
            rep = node.get("replacement", "▁")
            scheme = node.get("prepend_scheme", "always" if node.get("add_prefix_space", True) else "never")
            for i, p in enumerate(pieces):
                p = p.replace(" ", rep)
                if scheme == "always" or (scheme == "first" and i == 0):
                    if not p.startswith(rep):
                        p = rep + p
                if node.get("split", True):
                    out += [x for x in regex.split(f"(?={regex.escape(rep)})", p) if x]
                else:
                    out.append(p)
            return out
        if t in ("Whitespace", "WhitespaceSplit"):
            for p in pieces:
                out += regex.findall(r"\w+|[^\w\s]+", p) if t == "Whitespace" else p.split()
            return out
        raise ValueError(f"pre-tokenizer {t!r} is not supported")

    # ------------------------------------------------------------------ BPE
    def _bpe(self, piece: str) -> Tuple[int, ...]:
        if self.ignore_merges and piece in self.vocab:
            return (self.vocab[piece],)
        syms = list(piece)
        while len(syms) > 1:
            best, at = None, -1
            for i in range(len(syms) - 1):
                r = self.ranks.get((syms[i], syms[i + 1]))
                if r is not None and (best is None or r < best):
                    best, at = r, i
            if best is None:
                break
            syms[at:at + 2] = [syms[at] + syms[at + 1]]
        ids: List[int] = []
        unk_run = False
        for s in syms:
            if s in self.vocab:
                ids.append(self.vocab[s])
                unk_run = False
            elif self.byte_fallback:
                ids += [self.vocab[f"<0x{b:02X}>"] for b in s.encode("utf-8")]
                unk_run = False
            elif self.unk is not None:
                if not (self.fuse_unk and unk_run):
                    ids.append(self.vocab[self.unk])
                unk_run = True
            else:
                raise KeyError(f"symbol {s!r} is not in the vocabulary and no fallback is defined")
        return tuple(ids)

    def encode(self, text: str, add_special_tokens: bool = False) -> List[int]:
        ids: List[int] = []
        segments: List[Tuple[str, Optional[int]]] = []
        pos = 0
        if self._added_re is not None:
            for mt in self._added_re.finditer(text):
                if mt.start() > pos:
                    segments.append((text[pos:mt.start()], None))
                segments.append((mt.group(), self.added[mt.group()]))
                pos = mt.end()
        if pos < len(text):
            segments.append((text[pos:], None))
        for seg, sid in segments:
            if sid is not None:
                ids.append(sid)
                continue
            for piece in self._split([self._normalize(seg)], self.pre):
                ids += self._cache(piece)
        if add_special_tokens:
            ids = self._template(ids)
        return ids

    def _template(self, ids: List[int]) -> List[int]:
        node = self.post
        if not node:
            return ids
        if node.get("type") == "Sequence":
            for n in node.get("processors", []):
                if n.get("type") == "TemplateProcessing":
                    node = n
                    break
            else:
                return ids
        if node.get("type") != "TemplateProcessing":
            return ids
        out: List[int] = []
        for item in node.get("single", []):
            if "SpecialToken" in item:
                tok = item["SpecialToken"]["id"]
                out += node.get("special_tokens", {}).get(tok, {}).get("ids", [self.added.get(tok, self.vocab.get(tok))])
            elif "Sequence" in item:
                out += ids
        return out

    # ------------------------------------------------------------------ decode
    def decode(self, ids: Sequence[int], skip_special_tokens: bool = True) -> str:
        toks = [self.id_to_token.get(int(i), "") for i in ids
                if not (skip_special_tokens and int(i) in self.special_ids)]
        if self.byte_level:
            out = bytearray()
            for t in toks:
                if t in self.added:
                    out += t.encode("utf-8")
                else:
                    out += bytes(_U2B.get(c, ord("?")) for c in t)
            return out.decode("utf-8", "replace")
        buf = bytearray()
        for t in toks:
            if len(t) == 6 and t.startswith("<0x") and t.endswith(">"):
                buf.append(int(t[3:5], 16))
            else:
                buf += t.replace("▁", " ").encode("utf-8")
        s = buf.decode("utf-8", "replace")
        return s[1:] if s.startswith(" ") and self._strips_leading_space() else s

    def _strips_leading_space(self) -> bool:
        d = self.decoder or {}
        nodes = d.get("decoders", [d])
        return any(n.get("type") == "Strip" and n.get("start", 0) >= 1 for n in nodes) or \
            any(n.get("type") == "Metaspace" for n in nodes)
