"""Rewrite a launch YAML into the sectioned finetune layout, keeping comments.

    python -m deltaserve_vllm_b200.config_convert old.yaml            # print
    python -m deltaserve_vllm_b200.config_convert old.yaml -o new.yaml
    python -m deltaserve_vllm_b200.config_convert --in-place a.yaml b.yaml

The loader (``config_loader``) reads the legacy single ``finetune`` section
and keys placed in another finetune section than their own, with a note or a
warning each time. This tool moves every finetune key into its own section
(``finetune_param`` ... ``telemetry``, in that order, where the first
finetune section stood), drops retired keys, and copies every other section
as it is. It works on lines, not on a YAML round trip, so that comments
survive: a key moves together with the comment lines directly above it and
the more-indented lines of its value. The result must load to the same
finetune settings and engine keys as the input, or nothing is written.
The reference ships the same conversion for its own files
(``scripts/convert_config_layout.py``).
"""

from __future__ import annotations

import argparse
import re
import sys
from pathlib import Path

import yaml

from .config_loader import (ALL_FINETUNE_SECTIONS, FINETUNE_SECTIONS, RETIRED_KEYS, SECTION_OF, engine_kwargs,
                            finetune_kwargs)

_SECTION = re.compile(r"^([A-Za-z_][\w-]*)\s*:\s*(#.*)?$")
_KEY = re.compile(r"^(\s+)([A-Za-z_][\w-]*)\s*:")


def _split_sections(lines: list[str]) -> tuple[list[str], list[tuple[str, list[str], list[str]]]]:
    """(header lines, [(section name, lead lines, body lines)]): a section's
    lead lines are the comment lines directly above its header plus the
    header itself."""
    header: list[str] = []
    sections: list[tuple[str, list[str], list[str]]] = []
    pending: list[str] = []
    for line in lines:
        m = _SECTION.match(line)
        if m:
            lead = []
            # comment lines glued to the header (no blank line between) lead it
            while pending and pending[-1].strip().startswith("#"):
                lead.insert(0, pending.pop())
            (sections[-1][2] if sections else header).extend(pending)
            pending = []
            sections.append((m.group(1), lead + [line], []))
        else:
            pending.append(line)
    (sections[-1][2] if sections else header).extend(pending)
    return header, sections


def _split_entries(body: list[str]) -> tuple[list[tuple[str | None, list[str]]], list[str]]:
    """A section body as ([(key, lines)], trailing lines): each key keeps the
    comment lines directly above it and its more-indented continuation
    lines; blank lines between entries stay with the entry before them."""
    entries: list[tuple[str | None, list[str]]] = []
    base = None
    for line in body:
        m = _KEY.match(line)
        if m and not line.strip().startswith("#"):
            base = len(m.group(1)) if base is None else base
            if len(m.group(1)) == base:
                lead = []
                prev = entries[-1][1] if entries else None
                while prev and prev[-1].strip().startswith("#") and _indent(prev[-1]) <= base:
                    lead.insert(0, prev.pop())
                entries.append((m.group(2), lead + [line]))
                continue
        if entries:
            entries[-1][1].append(line)
        else:
            entries.append((None, [line]))
    trailing: list[str] = []
    if entries:
        lines = entries[-1][1]
        while lines and not lines[-1].strip():
            trailing.insert(0, lines.pop())
    return entries, trailing


def _indent(line: str) -> int:
    return len(line) - len(line.lstrip(" "))


def convert_text(text: str) -> tuple[str, list[str]]:
    """Converted YAML text and the notes (moved and dropped keys)."""
    lines = text.splitlines()
    header, sections = _split_sections(lines)
    notes: list[str] = []
    ft_lead: dict[str, list[str]] = {}
    ft_entries: dict[str, list[list[str]]] = {s: [] for s in FINETUNE_SECTIONS}
    loose: dict[str, list[list[str]]] = {}
    legacy_lead: list[str] = []
    first_ft = None
    for i, (name, lead, body) in enumerate(sections):
        if name not in ALL_FINETUNE_SECTIONS:
            continue
        first_ft = i if first_ft is None else first_ft
        if name in FINETUNE_SECTIONS:
            ft_lead[name] = lead
        else:                                 # comments above a legacy section header
            legacy_lead.extend(lead[:-1])
        entries, _ = _split_entries(body)
        for key, elines in entries:
            if key is None:                   # comments before the first key
                loose.setdefault(name if name in FINETUNE_SECTIONS else "finetune_param", []).append(elines)
                continue
            if key in RETIRED_KEYS:
                notes.append(f"dropped {name}.{key} ({RETIRED_KEYS[key]})")
                continue
            home = SECTION_OF.get(key)
            if home is None:
                raise ValueError(f"{name}.{key} is not a finetune setting")
            if home != name:
                notes.append(f"moved {name}.{key} -> {home}.{key}")
            ft_entries[home].append(elines)
    out: list[str] = list(header)
    for i, (name, lead, body) in enumerate(sections):
        if name in ALL_FINETUNE_SECTIONS:
            if i != first_ft:
                continue
            for sec in FINETUNE_SECTIONS:
                blocks = loose.get(sec, []) + ft_entries[sec]
                if not blocks:
                    continue
                if sec not in ft_lead:            # a new section: the legacy header's comments lead the first
                    out.extend(legacy_lead)
                    legacy_lead = []
                out.extend(ft_lead.get(sec, [f"{sec}:"]))
                for b in blocks:
                    out.extend(b)
                while out and not out[-1].strip():
                    out.pop()
                out.append("")
            continue
        out.extend(lead)
        out.extend(body)
    while out and not out[-1].strip():
        out.pop()
    return "\n".join(out) + "\n", notes


def _settings(text: str) -> tuple[dict, dict]:
    raw = yaml.safe_load(text) or {}
    for k in RETIRED_KEYS:
        for s in ALL_FINETUNE_SECTIONS:
            (raw.get(s) or {}).pop(k, None)
    import contextlib
    import io
    with contextlib.redirect_stdout(io.StringIO()):
        return finetune_kwargs(raw), engine_kwargs(raw)


def convert(text: str) -> tuple[str, list[str]]:
    """:func:`convert_text` plus the check that the result loads to the same
    finetune settings and engine keys as the input."""
    new, notes = convert_text(text)
    if _settings(new) != _settings(text):
        raise ValueError("the converted layout does not load to the same settings; nothing written")
    return new, notes


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("paths", nargs="+")
    ap.add_argument("-o", "--output", default=None, help="write here (one input only)")
    ap.add_argument("--in-place", action="store_true")
    a = ap.parse_args(argv)
    if a.output and len(a.paths) != 1:
        ap.error("-o takes one input")
    for p in a.paths:
        new, notes = convert(Path(p).read_text())
        for n in notes:
            print(f"[{p}] {n}", file=sys.stderr)
        if a.in_place:
            Path(p).write_text(new)
        elif a.output:
            Path(a.output).write_text(new)
        else:
            sys.stdout.write(new)


if __name__ == "__main__":
    main()
