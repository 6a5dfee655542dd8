def build_decoder(cfg, tp=None, device=None, pp=None):
    """The decoder class for a config: Gemma4LM for arch "gemma4", DecoderLM
    otherwise (pp: a pipeline stage, parallel.pipeline.PPInfo)."""
    if cfg.arch == "gemma4":
        if pp is not None and pp.stages > 1:
            raise ValueError("Gemma4 runs on one GPU")
        from .gemma4 import Gemma4LM

        return Gemma4LM(cfg, tp, device)
    from .llama import DecoderLM

    return DecoderLM(cfg, tp, device, pp=pp)
