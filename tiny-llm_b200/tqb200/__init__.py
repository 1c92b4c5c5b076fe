"""tqb200 — B200-native quantised decode hot path for tinyqwen (host-side package)."""
