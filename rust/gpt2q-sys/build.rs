// Links libgpt2q.so, built in-tree by `python -m smelt_b200.build` (smelt_b200/_lib/).
// GPT2Q_LIB_DIR overrides the location; the default is the library directory of this checkout.
fn main() {
    let dir = std::env::var("GPT2Q_LIB_DIR").unwrap_or_else(|_| {
        let here = std::env::var("CARGO_MANIFEST_DIR").expect("cargo sets CARGO_MANIFEST_DIR");
        format!("{here}/../../smelt_b200/_lib")
    });
    println!("cargo:rerun-if-env-changed=GPT2Q_LIB_DIR");
    println!("cargo:rustc-link-search=native={dir}");
    println!("cargo:rustc-link-lib=dylib=gpt2q");
    // let binaries find the library without LD_LIBRARY_PATH
    println!("cargo:rustc-link-arg=-Wl,-rpath,{dir}");
}
