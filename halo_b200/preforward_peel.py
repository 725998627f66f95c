"""Route long prompts of stock ``model.generate`` through chunked prefill
(``halo/preforward_peel.py`` in lzbaclz/HALO, :41-150)."""
from __future__ import annotations


def install_preforward_peel(model, *, prefill_chunk_tokens: int = 4096,
                            activation_threshold: int = 8192):
    """Patch ``model.generate`` (a model already wrapped with
    ``HALOConfig(chunked=True)``) so prompts longer than
    ``activation_threshold`` tokens run :func:`prefill_then_generate`.
    Raises ``ValueError`` otherwise; idempotent."""
    cfg = getattr(model, "_halo_config", None)
    if not cfg or not cfg.chunked:
        raise ValueError("install_preforward_peel requires a Path D / chunked HALO model. "
                         "Wrap first via wrap_with_halo(model, HALOConfig(chunked=True)).")
    if getattr(model, "_halo_preforward_patched", False):
        return model
    original = model.generate

    def generate(*args, **kwargs):
        ids = kwargs.get("input_ids", args[0] if args else None)
        if ids is None or ids.shape[-1] <= activation_threshold:
            return original(*args, **kwargs)
        from halo_b200.chunked_prefill import prefill_then_generate
        res = prefill_then_generate(model, ids, prefill_chunk_tokens=prefill_chunk_tokens,
                                    max_new_tokens=kwargs.get("max_new_tokens", 32),
                                    do_sample=kwargs.get("do_sample", False),
                                    temperature=kwargs.get("temperature", 1.0),
                                    top_p=kwargs.get("top_p", 1.0))
        return _PreforwardPeelResult(res["generated_ids"], res)

    model.generate = generate
    model._halo_preforward_patched = True
    model._halo_preforward_chunk = prefill_chunk_tokens
    model._halo_preforward_threshold = activation_threshold
    return model


class _PreforwardPeelResult:
    """Generate-like result: ``.sequences`` plus tensor-style indexing."""

    def __init__(self, sequences, telemetry: dict) -> None:
        self.sequences = sequences
        self.halo_telemetry = telemetry

    def __getitem__(self, idx):
        return self.sequences[idx]

    def __iter__(self):
        yield self.sequences

    @property
    def shape(self):
        return self.sequences.shape

    def __len__(self):
        return len(self.sequences)


__all__ = ["install_preforward_peel"]
