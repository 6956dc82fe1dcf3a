// build.rs for rustwood with the librwgpu backend: links librwgpu.so, found through
// RWGPU_LIB_DIR (the directory holding the library built by rustwood_b200/build.py), and
// records that directory as a run-time search path so the binary finds it without
// LD_LIBRARY_PATH. The reference's own build steps (if any) stay beside these lines.
fn main() {
    let dir = std::env::var("RWGPU_LIB_DIR").unwrap_or_else(|_| "rustwood_b200".to_string());
    println!("cargo:rustc-link-search=native={dir}");
    println!("cargo:rustc-link-lib=dylib=rwgpu");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{dir}");
    println!("cargo:rerun-if-env-changed=RWGPU_LIB_DIR");
}
