"""draftkv (B200 build) -- self-speculative decoding with a compressed-KV drafter."""
