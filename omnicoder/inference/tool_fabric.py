"""Tool and constraint fabric (reference src/omnicoder/inference/tool_fabric.py:1-91): one place
where generation and the reasoning controllers run inline tool calls, fuse verifier signals into
one margin, and turn the media a prompt refers to into facts of a symbolic state.

  invoke_tools_in_text(text)       every `<tool>name(arg)</tool>` call in `text` runs through the
                                   tool registry; the result follows the call as `<result>...</result>`
  combine_verifier_signals(s, w)   weighted mean of per-modality margins (z-scored ones through a
                                   sigmoid): the unified margin of the reasoning helpers
  analyze_inputs(prompt, ...)      file paths in the prompt with an image / video / audio extension
                                   go to caller-supplied analyzers (a detector returning labels, a
                                   transcriber returning text); their findings become facts of a
                                   SymbolicState whose rendered block can be put in front of the prompt

The reference calls fixed detector / tracker / speech tools by name and drops every failure
silently; here the analyzers are parameters (none is bundled: they need external weights), and a
failing analyzer is reported in the returned `errors` list.
"""
from __future__ import annotations

from typing import Callable

from ..reasoning.omega import SymbolicState, unified_margin
from .tools import ToolRegistry

IMAGE_EXT = (".png", ".jpg", ".jpeg", ".bmp", ".gif")
VIDEO_EXT = (".mp4", ".mov")
AUDIO_EXT = (".wav", ".mp3", ".flac", ".m4a")


def invoke_tools_in_text(text: str, registry: ToolRegistry | None = None) -> str:
    return (registry or ToolRegistry()).run_calls(text)


def combine_verifier_signals(signals: dict, weights: dict | None = None) -> float:
    return unified_margin(signals, weights)


def media_paths(prompt: str, max_paths: int = 4) -> list[str]:
    exts = IMAGE_EXT + VIDEO_EXT + AUDIO_EXT
    out = [t.strip("\"'(),;") for t in prompt.split()]
    return [t for t in out if t.lower().endswith(exts)][:max_paths]


def analyze_inputs(prompt: str, modes: str = "image,audio,video",
                   detect: Callable[[str], list[str]] | None = None,
                   track: Callable[[str], list[str]] | None = None,
                   transcribe: Callable[[str], str] | None = None) -> tuple[str, SymbolicState, list[str]]:
    """(rendered context, state, errors).  `detect(path)` / `track(path)` return object labels for an
    image / a video; `transcribe(path)` returns the speech in an audio file."""
    want = {m.strip() for m in modes.split(",") if m.strip()}
    state, errors = SymbolicState(), []
    for p in media_paths(prompt):
        low = p.lower()
        try:
            if low.endswith(IMAGE_EXT) and "image" in want and detect is not None:
                for lab in detect(p) or []:
                    state.apply(f"fact: {' '.join(str(lab).split())} present_in image {p}")
            elif low.endswith(VIDEO_EXT) and "video" in want and track is not None:
                for lab in track(p) or []:
                    state.apply(f"fact: {' '.join(str(lab).split())} present_in video {p}")
            elif low.endswith(AUDIO_EXT) and "audio" in want and transcribe is not None:
                txt = " ".join((transcribe(p) or "").split())      # one line: the state's DSL is line based
                if txt:
                    state.apply(f"fact: transcript of {p} = {txt}")
        except Exception as e:   # one failing analyzer does not stop the others; it is reported
            errors.append(f"{p}: {type(e).__name__}: {e}")
    return state.render_context(), state, errors
