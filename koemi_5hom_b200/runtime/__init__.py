from koemi_5hom_b200.runtime.fast_decode import (BatchDecoder, SamplingPolicy, TokenSampler, clone_state,
                                                 generate_tokens, to_static_state)

__all__ = ["BatchDecoder", "SamplingPolicy", "TokenSampler", "clone_state", "generate_tokens", "to_static_state"]
