#!/bin/sh
# ref_links.sh REF OUTDIR PATH... -- for each PATH (relative to REF) create
# OUTDIR/<name> -> REF/PATH where <name> is the literal string the reference
# writes in its quoted includes: "..\\dir\\file.h" (two backslashes per
# separator, as gcc does not unescape include names).
ref="$1"; out="$2"; shift 2
mkdir -p "$out"
for p in "$@"; do
  name="..$(printf '%s' "/$p" | sed 's#/#\\\\#g')"
  ln -sfn "$ref/$p" "$out/$name"
done
