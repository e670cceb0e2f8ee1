"""Chain-side crypto kernels of the reference's arc-gpu crate: BLAKE3 batch
transaction commitments + Merkle roots (``commit``), Ed25519 batch
signature verification (``ed25519``)."""
