"""CLI argument surface of the diffusion backends (no GPU): the video and
image-edit options parse and route to their runners."""
from bloom_b200.cli.infer import build_parser


def test_video_and_edit_arguments_parse():
    a = build_parser().parse_args(["--backend", "wan", "--model", "tiny-wan", "--prompt", "fox", "--width", "48",
                                   "--height", "32", "--num-frames", "5", "--num-steps", "2", "--guidance-scale",
                                   "3.5", "--negative-prompt", "blur", "--fps", "8", "-o", "x.gif"])
    assert (a.backend, a.width, a.height, a.num_frames, a.num_steps, a.guidance_scale, a.negative_prompt, a.fps,
            a.output) == ("wan", 48, 32, 5, 2, 3.5, "blur", 8.0, "x.gif")
    b = build_parser().parse_args(["--backend", "longcat", "--model", "tiny-longcat", "--image", "in.png", "-o",
                                   "out.png", "--prompt", "red"])
    assert (b.backend, b.image, b.output) == ("longcat", "in.png", "out.png")
