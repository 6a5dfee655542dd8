def build_decoder(cfg, tp=None, device=None):
    """The decoder class for a config: Gemma4LM for arch "gemma4", DecoderLM otherwise."""
    if cfg.arch == "gemma4":
        from .gemma4 import Gemma4LM

        return Gemma4LM(cfg, tp, device)
    from .llama import DecoderLM

    return DecoderLM(cfg, tp, device)
