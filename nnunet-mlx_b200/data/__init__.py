"""Raw-case preprocessing on the device (the step before the sliding window)."""
