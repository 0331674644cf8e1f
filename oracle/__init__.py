"""CPU oracle for the FlashMoE hot path: test infrastructure, never the product path."""
