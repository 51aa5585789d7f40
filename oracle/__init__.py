"""CPU oracle of the lm_head CE head: test infrastructure, never imported by the product path."""
