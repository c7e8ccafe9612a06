{
  "targets": [
    {
      "target_name": "gsampler",
      "sources": ["gsampler_napi.cc"],
      "include_dirs": ["<(module_root_dir)/../../include"],
      "cflags_cc": ["-std=c++17", "-O2"],
      "libraries": ["-L<(module_root_dir)/..", "-lgsampler", "-Wl,-rpath,<(module_root_dir)/.."]
    }
  ]
}
