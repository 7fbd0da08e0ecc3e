"""nyion.rs_b200 — B200-native attention hot path of bmcc-DEV/Nyion.rs."""
