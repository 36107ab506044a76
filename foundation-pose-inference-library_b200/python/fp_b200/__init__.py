"""Python helpers of the FoundationPose B200 runtime: fpk kernel bindings,
network weight packs and seeded synthetic scenes."""
